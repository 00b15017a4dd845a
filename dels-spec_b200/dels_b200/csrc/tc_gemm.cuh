// Persistent warp-specialised tcgen05 GEMM with two epilogues (sm_100a).
//
//   D[m, n] = sum_k A[m, k] * B[n, k]        A, B bf16 K-major, D fp32 in TMEM
//
// The K range is the concatenation of two segments, each with its own pair of TMA
// maps: segment 0 (A0, B0) for kb0 k-blocks, then segment 1 (A1, B1) for kb1
// k-blocks.  The draft-scoring kernel uses this to fold both contractions of
//
//   score[row, v] = sum_k h[row, k] W[v, k]  +  alpha_p * sum_j s[row, j] Vr[v, j]
//
// into ONE accumulator: segment 0 is (h, W) over H, segment 1 is (alpha_p * s, Vr)
// over r (the per-row alpha is folded into the bf16 rank state before the call).
// Reference: code/kernel/dels.py:49-79 (the low-rank part) and code/dflash.py:468 (the
// long-logit GEMM, which the reference materialises and this kernel does not).
//
// Tile: 128 rows (TMEM lanes) x BN columns (TMEM columns), 64-element K blocks staged
// by TMA into 128-byte-swizzled shared memory, accumulators double-buffered in TMEM
// so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA
// issuer (one thread), warps 2..5 = epilogue (one thread per accumulator row).
//
// Epilogues:
//   kArgmax : score = acc (+ base[row, v]) - beta_p * prior[v]; the packed (score,
//             index) key of each 32-column chunk (chunk_best_key) folded into a running
//             maximum in registers, then one 64-bit atomicMax per (row, tile).  The last CTA to finish decodes the
//             keys into int64 token ids (optional).
//   kStore  : write the fp32 accumulator tile to out[split][row][n] (split-K partial
//             sums; used by the rank projection and the RNN input projection), or, with
//             out_bf16 set (one K split), bf16(acc + bias[n]) straight to out_bf16[row][n]
//             (F.linear with a bf16 result, e.g. the long logits h . W^T of
//             code/dflash.py:468).
#pragma once

#include "common.cuh"

namespace dels {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kTcThreads = 192;

enum TcEpilogue { kArgmax = 0, kStore = 1 };

struct TcArgs {
  int m_rows;              // rows of A (capacity)
  const int* m_rows_dev;   // optional device-side row count (clamped to m_rows)
  int n_cols;              // rows of B (vocab slice length, or r for the projection)
  int kb0, kb1;            // k-blocks in segment 0 and segment 1
  int k_splits;            // split-K factor (kStore only; 1 for kArgmax)
  int kb_per_split;
  int group_m;             // rasterisation: row tiles that sweep the B operand together
  int tail_split;          // the last partial wave's tiles are split this many ways along N
  int* status;             // device error word (0 = ok)
  // kArgmax
  long long v_begin;       // global vocab index of column 0 of B
  const float* prior;      // [n_cols] fp32 or null (beta term skipped)
  const float* beta;       // [n_pos]
  const int* row_pos;      // [m_rows] position of each row, or null (row % n_pos)
  int n_pos;
  const __nv_bfloat16* base;  // base logits: base[row * ld_base + v] or null
  long long ld_base;
  long long* keys;         // [m_rows] packed keys, pre-filled with kKeyEmpty
  long long* idx_out;      // [m_rows] decoded token ids, or null (keys are left for a combine)
  float* score_out;        // [m_rows] winning scores, or null
  unsigned* counter;       // zero on entry; the last CTA resets it
  // kStore
  float* out;
  long long ld_out;
  long long split_stride;
  __nv_bfloat16* out_bf16;         // non-null: bf16 result (k_splits == 1), row stride ld_out
  const __nv_bfloat16* bias_bf16;  // [n_cols] or null (out_bf16 only)
  int out_vec;                     // out_bf16 and ld_out allow 16-byte stores
  // skinny scorer with helper warps (tc_skinny_gh_kernel): the next rollout step's
  // gh_out[b] = bf16(gh_w . gh_x[b] + gh_bias), beside the scoring pipeline
  const __nv_bfloat16* gh_w;     // [gh_rows, gh_k]
  const __nv_bfloat16* gh_bias;  // [gh_rows] or null
  const __nv_bfloat16* gh_x;     // [gh_b, gh_k]
  __nv_bfloat16* gh_out;         // [gh_b, gh_rows]
  int gh_rows, gh_k, gh_b;
};

// STAGED: the argmax epilogue with base logits prefetches each tile's base rows and
// prior slice into shared memory (one region per epilogue warp) before it waits for
// the accumulator, so their load latency overlaps the tile's MMAs instead of being
// paid once per 32-column chunk.  It gives up one operand stage for the room.
template <int BN, bool STAGED = false>
struct TcConfig {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = STAGED ? 3 : ((BN >= 256) ? 4 : (BN >= 128 ? 6 : 8));
  static constexpr int kAccCols = 2 * BN;
  static constexpr int kTmemCols =
      kAccCols <= 32 ? 32 : (kAccCols <= 64 ? 64 : (kAccCols <= 128 ? 128 : (kAccCols <= 256 ? 256 : 512)));
  // per epilogue warp: 32 rows of BN bf16, each padded by 16 bytes so that the
  // lane-per-row 16-byte reads of a quarter warp hit distinct banks, and BN fp32 prior
  static constexpr int kBaseLd = BN + 8;
  static constexpr int kBaseWarpBytes = 32 * kBaseLd * 2;
  static constexpr int kPriorWarpBytes = BN * 4;
  static constexpr int kEpiOffset = kStages * kStageBytes;
  static constexpr int kEpiBytes = STAGED ? 4 * (kBaseWarpBytes + kPriorWarpBytes) : 0;
  static constexpr int kBarOffset = kEpiOffset + kEpiBytes;
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// One 32-column chunk of an accumulator row as bf16(0 + acc + bias): the same value (and
// sign of zero) as the split-K finalisation of a single split.  dst and bias point at the
// chunk's first column; `valid` columns are written; vec: 16-byte aligned dst and bias.
__device__ __forceinline__ void store_chunk_bf16(const uint32_t (&v)[32], int valid, __nv_bfloat16* dst,
                                                 const __nv_bfloat16* bias, int vec) {
  float x[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = 0.0f + __uint_as_float(v[j]);
  if (vec && valid >= 32) {
    if (bias != nullptr) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias) + q);
        x[8 * q + 0] += bf16_lo(w.x);
        x[8 * q + 1] += bf16_hi(w.x);
        x[8 * q + 2] += bf16_lo(w.y);
        x[8 * q + 3] += bf16_hi(w.y);
        x[8 * q + 4] += bf16_lo(w.z);
        x[8 * q + 5] += bf16_hi(w.z);
        x[8 * q + 6] += bf16_lo(w.w);
        x[8 * q + 7] += bf16_hi(w.w);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 o;
      o.x = pack_bf16x2(x[8 * q + 0], x[8 * q + 1]);
      o.y = pack_bf16x2(x[8 * q + 2], x[8 * q + 3]);
      o.z = pack_bf16x2(x[8 * q + 4], x[8 * q + 5]);
      o.w = pack_bf16x2(x[8 * q + 6], x[8 * q + 7]);
      reinterpret_cast<uint4*>(dst)[q] = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) {
        float y = x[j];
        if (bias != nullptr) y += __bfloat162float(bias[j]);
        dst[j] = __float2bfloat16_rn(y);
      }
  }
}

struct TileCoord {
  int m_tile, n_tile, split;
};

// Tile t -> (row tile, column tile, K split).  Row tiles are taken in groups of
// group_m: a group sweeps every column tile with its row tiles fastest, so the group's
// A panel stays resident in L2 while the B operand (the LM head) streams through once
// per group, and CTAs that run concurrently share each B tile.
__device__ __forceinline__ TileCoord tile_coord(int t, int num_m, int num_n, int k_splits, int group_m) {
  TileCoord c;
  c.split = t % k_splits;
  const int mn = t / k_splits;
  const int per_group = group_m * num_n;
  const int g = mn / per_group;
  const int first_m = g * group_m;
  const int gm = min(group_m, num_m - first_m);
  const int local = mn - g * per_group;
  c.m_tile = first_m + local % gm;
  c.n_tile = local / gm;
  return c;
}

// Work unit u of the persistent schedule.  The first `main_units` units are whole
// tiles; the remaining tiles of the last, partial wave are split `tail_split` ways
// along N so that the wave's work spreads over all CTAs instead of a handful.
struct WorkUnit {
  TileCoord c;
  int n0;   // first B row (column of D) of the unit
  int bn;   // columns in this unit (BN or BN / tail_split)
  bool tail;
};

struct Schedule {
  int num_m, num_n, k_splits, group_m;
  int main_units, tail_split, total_units;
};

__device__ __forceinline__ Schedule make_schedule(int num_m, int num_n, int k_splits, int group_m, int tail_split,
                                                  int grid) {
  Schedule s;
  s.num_m = num_m;
  s.num_n = num_n;
  s.k_splits = k_splits;
  s.group_m = group_m < 1 ? 1 : group_m;
  const int tiles = num_m * num_n * k_splits;
  const int rem = grid > 0 ? tiles % grid : 0;
  s.tail_split = (tail_split > 1 && rem > 0) ? tail_split : 1;
  s.main_units = tiles - (s.tail_split > 1 ? rem : 0);
  s.total_units = s.main_units + (tiles - s.main_units) * s.tail_split;
  return s;
}

template <int BN>
__device__ __forceinline__ WorkUnit work_unit(int u, const Schedule& s) {
  WorkUnit w;
  if (u < s.main_units) {
    w.c = tile_coord(u, s.num_m, s.num_n, s.k_splits, s.group_m);
    w.n0 = w.c.n_tile * BN;
    w.bn = BN;
    w.tail = false;
  } else {
    const int q = u - s.main_units;
    w.c = tile_coord(s.main_units + q / s.tail_split, s.num_m, s.num_n, s.k_splits, s.group_m);
    w.bn = BN / s.tail_split;
    w.n0 = w.c.n_tile * BN + (q % s.tail_split) * w.bn;
    w.tail = true;
  }
  return w;
}

template <int BN, int MODE, bool VEC_BASE>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                   const __grid_constant__ CUtensorMap map_a1, const __grid_constant__ CUtensorMap map_b1,
                   const __grid_constant__ CUtensorMap map_b0t, const __grid_constant__ CUtensorMap map_b1t,
                   const TcArgs args) {
  constexpr bool STAGED = VEC_BASE && MODE == kArgmax;
  using Cfg = TcConfig<BN, STAGED>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];

  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);
  const uint32_t a_base = base_addr;
  const uint32_t b_base = base_addr + S * Cfg::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * S + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * S + 2 + a]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4 * 32);
    }
    *abort_flag = 0;
    *last_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&map_a0);
    tma_prefetch_map(&map_b0);
    tma_prefetch_map(&map_a1);
    tma_prefetch_map(&map_b1);
    tma_prefetch_map(&map_b0t);
    tma_prefetch_map(&map_b1t);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Set-up above touches no global memory; from here on the inputs of earlier kernels
  // (rows, keys, device row count) are read.
  pdl_wait();
  int m_rows = args.m_rows;
  if (args.m_rows_dev != nullptr) {
    const int d = *args.m_rows_dev;
    m_rows = d < 0 ? 0 : (d < m_rows ? d : m_rows);
  }
  const int num_m = (m_rows + kBM - 1) / kBM;
  const int num_n = (args.n_cols + BN - 1) / BN;
  const int total_kb = args.kb0 + args.kb1;
  const Schedule sched = make_schedule(num_m, num_n, args.k_splits, args.group_m, args.tail_split, gridDim.x);
  const int num_units = sched.total_units;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const WorkUnit wu = work_unit<BN>(u, sched);
        const int kb_begin = wu.c.split * args.kb_per_split;
        const int kb_end = min(total_kb, kb_begin + args.kb_per_split);
        const int m0 = wu.c.m_tile * kBM;
        const int n0 = wu.n0;
        const uint32_t tx = (uint32_t)Cfg::kABytes + (uint32_t)wu.bn * kBK * 2u;
        const CUtensorMap* mb0 = wu.tail ? &map_b0t : &map_b0;
        const CUtensorMap* mb1 = wu.tail ? &map_b1t : &map_b1;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), tx);
          const uint32_t a_dst = a_base + stage * Cfg::kABytes;
          const uint32_t b_dst = b_base + stage * Cfg::kBBytes;
          if (kb < args.kb0) {
            tma_load_2d(a_dst, &map_a0, full_bar(stage), kb * kBK, m0);
            tma_load_2d(b_dst, mb0, full_bar(stage), kb * kBK, n0);
          } else {
            const int k1 = kb - args.kb0;
            tma_load_2d(a_dst, &map_a1, full_bar(stage), k1 * kBK, m0);
            tma_load_2d(b_dst, mb1, full_bar(stage), k1 * kBK, n0);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Aborting: let the copies already in flight land before the CTA exits.
        const int outstanding = issued < S ? issued : S;
        int s = stage;
        uint32_t p = phase;
        for (int i = 0; i < outstanding; ++i) {
          if (--s < 0) {
            s = S - 1;
            p ^= 1u;
          }
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(full_bar(s), p) && globaltimer_ns() - t0 < kWaitLimitNs / 20) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_full = make_idesc_bf16_f32(kBM, BN);
      const uint32_t idesc_tail = make_idesc_bf16_f32(kBM, BN / (sched.tail_split > 1 ? sched.tail_split : 1));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const WorkUnit wu = work_unit<BN>(u, sched);
        const TileCoord tc = wu.c;
        const uint32_t idesc = wu.tail ? idesc_tail : idesc_full;
        const int kb_begin = tc.split * args.kb_per_split;
        const int kb_end = min(total_kb, kb_begin + args.kb_per_split);
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(a_base + stage * Cfg::kABytes);
          const uint64_t bdesc = make_sw128_desc(b_base + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzled row.
            tc_mma_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                        (kb > kb_begin || k > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(stage));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit(tfull_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: wait until every MMA this thread issued has completed before TMEM is
      // released (the normal path has already observed this through tfull).
      if (!ok || *abort_flag) {
        const uint32_t drain = tfull_bar(acc);
        tc_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, acc_phase) && globaltimer_ns() - t0 < kWaitLimitNs / 20) {
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp can access
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    // STAGED: this warp's base rows and prior slice in shared memory
    const int epi_slot = warp - 2;
    uint8_t* base_s = smem + Cfg::kEpiOffset + epi_slot * (Cfg::kBaseWarpBytes + Cfg::kPriorWarpBytes);
    const float* prior_s = reinterpret_cast<const float*>(base_s + Cfg::kBaseWarpBytes);
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const WorkUnit wu = work_unit<BN>(u, sched);
      const TileCoord tc = wu.c;
      const int row = tc.m_tile * kBM + row_in_tile;
      const bool row_ok = row < m_rows;
      const int n0 = wu.n0;
      const int ncols = min(wu.bn, args.n_cols - n0);
      const int nchunks = wu.bn / 32;
      // A warp whose 32 rows are all past the end skips the tile (warp-uniform, so the
      // collective tensor-memory loads stay aligned); lanes past the end skip the arithmetic.
      const int warp_row0 = tc.m_tile * kBM + quad * 32;
      const bool warp_rows = warp_row0 < m_rows;
      if constexpr (STAGED) {
        if (warp_rows) {
          // Row by row, each row's slice one coalesced warp-wide copy (lane l takes
          // elements 8l..8l+7 of every 256); the partial last 16 bytes are zero-filled.
          __syncwarp();  // every lane has finished reading the previous tile's copy
          const uint32_t dst0 = smem_u32(base_s);
          const int nr = min(32, m_rows - warp_row0);
          for (int rr = 0; rr < nr; ++rr) {
            const __nv_bfloat16* src = args.base + (long long)(warp_row0 + rr) * args.ld_base + n0;
            for (int e = lane * 8; e < ncols; e += 256)
              cp_async_16(dst0 + (uint32_t)((rr * Cfg::kBaseLd + e) * 2), src + e, (uint32_t)min(16, (ncols - e) * 2));
          }
          if (args.prior != nullptr) {
            const uint32_t pdst = smem_u32(prior_s);
            for (int e = lane * 4; e < ncols; e += 128)
              cp_async_16(pdst + (uint32_t)(e * 4), args.prior + n0 + e, (uint32_t)min(16, (ncols - e) * 4));
          }
          cp_async_commit();
        }
      }
      if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag, args.status)) {
        if constexpr (STAGED) cp_async_wait_all();
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);

      if constexpr (MODE == kArgmax) {
        float negb = 0.0f;
        if (row_ok && args.prior != nullptr)
          negb = -__ldg(&args.beta[row_position(args.row_pos, row, args.n_pos)]);
        const __nv_bfloat16* brow =
            (args.base != nullptr && row_ok) ? args.base + (long long)row * args.ld_base + n0 : nullptr;
        const float* prow = args.prior != nullptr ? args.prior + n0 : nullptr;
        const __nv_bfloat16* brow_s = reinterpret_cast<const __nv_bfloat16*>(base_s) + lane * Cfg::kBaseLd;
        if constexpr (STAGED) {
          cp_async_wait_all();
          __syncwarp();
        }
        long long best_key = kKeyEmpty;
        // the row's best score so far on the device: chunk_fold skips chunks below it
        float thr = row_ok ? key_threshold(__ldcg(&args.keys[row])) : -__int_as_float(0x7f800000);
#pragma unroll 1
        for (int c = 0; c < (warp_rows ? nchunks : 0); ++c) {
          uint32_t v[32];
          tmem_ld_32cols(t_row + (uint32_t)(c * 32), v);
          tmem_ld_wait(v);
          const int c0 = c * 32;
          if (row_ok && c0 < ncols) {
            float sc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) sc[j] = __uint_as_float(v[j]);
            const bool full_chunk = (c0 + 32 <= ncols);
            if constexpr (STAGED) {
              // staged operands; columns past ncols hold stale data and are masked in the scan
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 w = reinterpret_cast<const uint4*>(brow_s + c0)[q];
                sc[8 * q + 0] += bf16_lo(w.x);
                sc[8 * q + 1] += bf16_hi(w.x);
                sc[8 * q + 2] += bf16_lo(w.y);
                sc[8 * q + 3] += bf16_hi(w.y);
                sc[8 * q + 4] += bf16_lo(w.z);
                sc[8 * q + 5] += bf16_hi(w.z);
                sc[8 * q + 6] += bf16_lo(w.w);
                sc[8 * q + 7] += bf16_hi(w.w);
              }
              if (prow != nullptr) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  const float4 p = reinterpret_cast<const float4*>(prior_s + c0)[q];
                  // two packed two-lane FMAs: the rounding of four fmaf
                  const float2 lo = __ffma2_rn(make_float2(negb, negb), make_float2(p.x, p.y),
                                               make_float2(sc[4 * q + 0], sc[4 * q + 1]));
                  const float2 hi = __ffma2_rn(make_float2(negb, negb), make_float2(p.z, p.w),
                                               make_float2(sc[4 * q + 2], sc[4 * q + 3]));
                  sc[4 * q + 0] = lo.x;
                  sc[4 * q + 1] = lo.y;
                  sc[4 * q + 2] = hi.x;
                  sc[4 * q + 3] = hi.y;
                }
              }
            } else {
              if (brow != nullptr) {
                if (VEC_BASE && full_chunk) {
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const uint4 w = __ldg(reinterpret_cast<const uint4*>(brow + c0) + q);
                    sc[8 * q + 0] += bf16_lo(w.x);
                    sc[8 * q + 1] += bf16_hi(w.x);
                    sc[8 * q + 2] += bf16_lo(w.y);
                    sc[8 * q + 3] += bf16_hi(w.y);
                    sc[8 * q + 4] += bf16_lo(w.z);
                    sc[8 * q + 5] += bf16_hi(w.z);
                    sc[8 * q + 6] += bf16_lo(w.w);
                    sc[8 * q + 7] += bf16_hi(w.w);
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (c0 + j < ncols) sc[j] += __bfloat162float(brow[c0 + j]);
                }
              }
              if (prow != nullptr) {
                if (full_chunk) {
#pragma unroll
                  for (int q = 0; q < 8; ++q) {
                    const float4 p = __ldg(reinterpret_cast<const float4*>(prow + c0) + q);
                    // two packed two-lane FMAs: the rounding of four fmaf
                    const float2 lo = __ffma2_rn(make_float2(negb, negb), make_float2(p.x, p.y),
                                                 make_float2(sc[4 * q + 0], sc[4 * q + 1]));
                    const float2 hi = __ffma2_rn(make_float2(negb, negb), make_float2(p.z, p.w),
                                                 make_float2(sc[4 * q + 2], sc[4 * q + 3]));
                    sc[4 * q + 0] = lo.x;
                    sc[4 * q + 1] = lo.y;
                    sc[4 * q + 2] = hi.x;
                    sc[4 * q + 3] = hi.y;
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (c0 + j < ncols) sc[j] = fmaf(negb, __ldg(prow + c0 + j), sc[j]);
                }
              }
            }
            chunk_fold(sc, ncols - c0, (uint32_t)(args.v_begin + n0 + c0), best_key, thr);
          }
        }
        tc_fence_before();
        mbar_arrive(tempty_bar(acc));
        if (row_ok && best_key != kKeyEmpty) {  // empty: every chunk fell below the row's best
          atomicMax(&args.keys[row], best_key);
          __threadfence();
        }
      } else if (args.out_bf16 != nullptr) {
        __nv_bfloat16* dst = args.out_bf16 + (long long)row * args.ld_out + n0;
        const __nv_bfloat16* bias = args.bias_bf16 != nullptr ? args.bias_bf16 + n0 : nullptr;
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
          uint32_t v[32];
          tmem_ld_32cols(t_row + (uint32_t)(c * 32), v);
          tmem_ld_wait(v);
          const int c0 = c * 32;
          if (row_ok && c0 < ncols)
            store_chunk_bf16(v, ncols - c0, dst + c0, bias != nullptr ? bias + c0 : nullptr, args.out_vec);
        }
        tc_fence_before();
        mbar_arrive(tempty_bar(acc));
      } else {
        float* dst = args.out + (long long)tc.split * args.split_stride + (long long)row * args.ld_out + n0;
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
          uint32_t v[32];
          tmem_ld_32cols(t_row + (uint32_t)(c * 32), v);
          tmem_ld_wait(v);
          const int c0 = c * 32;
          if (row_ok && c0 < ncols) {
            if (c0 + 32 <= ncols) {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 f;
                f.x = __uint_as_float(v[4 * q + 0]);
                f.y = __uint_as_float(v[4 * q + 1]);
                f.z = __uint_as_float(v[4 * q + 2]);
                f.w = __uint_as_float(v[4 * q + 3]);
                reinterpret_cast<float4*>(dst + c0)[q] = f;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (c0 + j < ncols) dst[c0 + j] = __uint_as_float(v[j]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(tempty_bar(acc));
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }

  if constexpr (MODE == kArgmax) {
    if (args.idx_out != nullptr) {
      // The last CTA to finish turns the packed keys into token ids.
      if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(args.counter, 1u);
        *last_flag = (prev == gridDim.x - 1) ? 1 : 0;
      }
      __syncthreads();
      if (*last_flag) {
        __threadfence();
        for (int row = threadIdx.x; row < m_rows; row += blockDim.x) {
          const long long key = (long long)atomicAdd(reinterpret_cast<unsigned long long*>(&args.keys[row]), 0ull);
          args.idx_out[row] = (long long)key_index(key);
          if (args.score_out != nullptr) args.score_out[row] = key_score(key);
        }
        if (threadIdx.x == 0) atomicExch(args.counter, 0u);
      }
    }
  }
}

}  // namespace dels
