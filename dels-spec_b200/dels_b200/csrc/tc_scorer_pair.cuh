// Fused draft scorer on CTA pairs: tcgen05.mma.cta_group::2, M = 256 rows per pair tile.
//
// Same contraction, epilogue and schedule as tc_gemm_kernel<256, kArgmax> (see
// tc_gemm.cuh), reorganised around 2-CTA clusters so that each SM streams only HALF of
// every 256-token LM-head tile:
//
//   pair tile = 256 rows x BN vocabulary columns; CTA rank c of the pair owns rows
//   [m0 + 128c, m0 + 128c + 128) (its A tile) and vocabulary rows
//   [n0 + c*BN/2, n0 + (c+1)*BN/2) of the B tile.  The MMA issued by rank 0 reads A and
//   B from both CTAs' shared memory at the same offsets and writes each CTA's 128-row
//   half of the fp32 accumulator into that CTA's tensor memory.
//
// Per SM and per 64-wide K block this moves 16 KB of A + 16 KB of B through shared
// memory for 128 x 256 x 64 MACs, against 16 + 32 KB in the single-CTA kernel, so the
// shared-memory traffic per tensor-core FLOP drops by a third and the ring gets six
// slots instead of four.  With KG = 2 two adjacent slots form one pipeline stage: the
// producer fetches both K blocks of every W row together (256 contiguous bytes per row
// instead of 128 bytes one stage apart), which streams the LM head from HBM faster
// (a TMA probe of this kernel's access pattern: 5.5 against 4.5 TB/s).
//
// Synchronisation (all barriers live at the same offsets in both CTAs):
//   full[s]   rank 0 only: one arrive.expect_tx for both CTAs' bytes; both CTAs' TMA
//             loads complete_tx on it (cta_group::2 TMA, rank 0's barrier address)
//   empty[s]  both CTAs: the MMA's commit arrives on both (multicast over the pair)
//   tfull[a]  both CTAs: the MMA's commit at the end of a tile arrives on both
//   tempty[a] rank 0 only: 4 epilogue-warp arrivals from each CTA (peer arrives remotely)
// A cluster barrier after set-up (peer barriers initialised) and before teardown (no
// CTA exits while its partner may still touch its shared memory) brackets the loops.
// Every mbarrier wait is bounded as in tc_gemm.cuh.
#pragma once

#include "tc_gemm.cuh"

namespace dels {

struct PairConfig {
  static constexpr int BN = 256;           // vocabulary columns per pair tile
  static constexpr int kHalfBN = BN / 2;   // B rows staged by each CTA
  static constexpr int kABytes = kBM * kBK * 2;        // 16 KB
  static constexpr int kBBytes = kHalfBN * kBK * 2;    // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 6;
  static constexpr int kTmemCols = 512;                // two 256-column accumulators
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// STORE: instead of the argmax, write each accumulator row as bf16 to args.out_bf16
// (store_chunk_bf16; the long logits h . W^T when a caller wants them materialised).
template <bool VEC_BASE, bool STORE = false, int KG = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    tc_scorer_pair_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                          const __grid_constant__ CUtensorMap map_a1, const __grid_constant__ CUtensorMap map_b1,
                          const __grid_constant__ CUtensorMap map_b0t, const __grid_constant__ CUtensorMap map_b1t,
                          const TcArgs args) {
  using Cfg = PairConfig;
  constexpr int S = Cfg::kStages;  // shared-memory slots, one K block each
  static_assert(KG == 1 || KG == 2, "K blocks per pipeline stage");
  constexpr int SG = S / KG;        // pipeline stages (groups of KG slots)
  constexpr int BN = Cfg::BN;
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SG; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps in each CTA of the pair
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
    tmem_alloc_pair(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
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
  const int num_m = (m_rows + 2 * kBM - 1) / (2 * kBM);  // pair tiles along the rows
  const int num_n = (args.n_cols + BN - 1) / BN;
  const int total_kb = args.kb0 + args.kb1;
  const Schedule sched = make_schedule(num_m, num_n, 1, args.group_m, args.tail_split, num_pairs);
  const int num_units = sched.total_units;


  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += num_pairs) {
        const WorkUnit wu = work_unit<BN>(u, sched);
        const int m0 = wu.c.m_tile * 2 * kBM + (int)rank * kBM;
        const int half = wu.bn / 2;
        const int n0 = wu.n0 + (int)rank * half;
        const uint32_t tx_pair = 2u * ((uint32_t)Cfg::kABytes + (uint32_t)half * kBK * 2u);
        const CUtensorMap* mb0 = wu.tail ? &map_b0t : &map_b0;
        const CUtensorMap* mb1 = wu.tail ? &map_b1t : &map_b1;
        for (int kb = 0; kb < total_kb; kb += KG) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          const int nb = total_kb - kb < KG ? total_kb - kb : KG;  // K blocks in this stage
          const uint32_t full_leader = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), tx_pair * (uint32_t)nb);
          for (int j = 0; j < nb; ++j) {
            const int slot = stage * KG + j, kj = kb + j;
            const uint32_t a_dst = a_base + slot * Cfg::kABytes;
            const uint32_t b_dst = b_base + slot * Cfg::kBBytes;
            if (kj < args.kb0) {
              tma_load_2d_pair(a_dst, &map_a0, full_leader, kj * kBK, m0);
              tma_load_2d_pair(b_dst, mb0, full_leader, kj * kBK, n0);
            } else {
              const int k1 = kj - args.kb0;
              tma_load_2d_pair(a_dst, &map_a1, full_leader, k1 * kBK, m0);
              tma_load_2d_pair(b_dst, mb1, full_leader, k1 * kBK, n0);
            }
          }
          ++issued;
          if (++stage == SG) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Aborting: the copies in flight complete on rank 0's full barriers; rank 0
        // drains them, the peer waits out the same bounded delay before leaving.
        const unsigned long long t0 = globaltimer_ns();
        int s = stage;
        uint32_t p = phase;
        const int outstanding = issued < SG ? issued : SG;
        for (int i = 0; i < outstanding && leader; ++i) {
          if (--s < 0) {
            s = SG - 1;
            p ^= 1u;
          }
          while (!mbar_try_wait(full_bar(s), p) && globaltimer_ns() - t0 < kWaitLimitNs / 20) {
          }
        }
        while (!leader && globaltimer_ns() - t0 < kWaitLimitNs / 40) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (rank 0)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc_full = make_idesc_bf16_f32(2 * kBM, BN);
      const uint32_t idesc_tail = make_idesc_bf16_f32(2 * kBM, BN / (sched.tail_split > 1 ? sched.tail_split : 1));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += num_pairs) {
        const WorkUnit wu = work_unit<BN>(u, sched);
        const uint32_t idesc = wu.tail ? idesc_tail : idesc_full;
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < total_kb; kb += KG) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nb = total_kb - kb < KG ? total_kb - kb : KG;
          for (int j = 0; j < nb; ++j) {
            const int slot = stage * KG + j;
            const uint64_t adesc = make_sw128_desc(a_base + slot * Cfg::kABytes);
            const uint64_t bdesc = make_sw128_desc(b_base + slot * Cfg::kBBytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              tc_mma_pair_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                               (kb + j > 0 || k > 0) ? 1u : 0u);
            }
          }
          tc_commit_pair_both(empty_bar(stage));
          if (++stage == SG) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit_pair_both(tfull_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok || *abort_flag) {
        const uint32_t drain = tfull_bar(acc);
        tc_commit_pair_both(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, acc_phase) && globaltimer_ns() - t0 < kWaitLimitNs / 20) {
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;
    const int row_in_tile = (int)rank * kBM + quad * 32 + lane;
    const uint32_t tempty_leader0 = mapa_shared(tempty_bar(0), 0);
    const uint32_t tempty_leader1 = mapa_shared(tempty_bar(1), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < num_units; u += num_pairs) {
      const WorkUnit wu = work_unit<BN>(u, sched);
      const int row = wu.c.m_tile * 2 * kBM + row_in_tile;
      const bool row_ok = row < m_rows;
      const int n0 = wu.n0;
      const int ncols = min(wu.bn, args.n_cols - n0);
      const int nchunks = wu.bn / 32;
      if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      // A warp whose 32 rows are all past the end skips the tile (warp-uniform, so the
      // collective tensor-memory loads stay aligned); lanes past the end skip the
      // arithmetic.
      const bool warp_rows = (wu.c.m_tile * 2 * kBM + (int)rank * kBM + quad * 32) < m_rows;

      if constexpr (STORE) {
        __nv_bfloat16* dst = args.out_bf16 + (long long)row * args.ld_out + n0;
        const __nv_bfloat16* bias = args.bias_bf16 != nullptr ? args.bias_bf16 + n0 : nullptr;
#pragma unroll 1
        for (int c = 0; c < (warp_rows ? nchunks : 0); ++c) {
          uint32_t v[32];
          tmem_ld_32cols(t_row + (uint32_t)(c * 32), v);
          tmem_ld_wait(v);
          const int c0 = c * 32;
          if (row_ok && c0 < ncols)
            store_chunk_bf16(v, ncols - c0, dst + c0, bias != nullptr ? bias + c0 : nullptr, args.out_vec);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(tempty_bar(acc));
          else
            mbar_arrive_remote(acc == 0 ? tempty_leader0 : tempty_leader1);
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
        continue;
      }

      float negb = 0.0f;
      if (row_ok && args.prior != nullptr) negb = -__ldg(&args.beta[row_position(args.row_pos, row, args.n_pos)]);
      const __nv_bfloat16* brow =
          (args.base != nullptr && row_ok) ? args.base + (long long)row * args.ld_base + n0 : nullptr;
      const float* prow = args.prior != nullptr ? args.prior + n0 : nullptr;
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
          chunk_fold(sc, ncols - c0, (uint32_t)(args.v_begin + n0 + c0), best_key, thr);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(tempty_bar(acc));
        else
          mbar_arrive_remote(acc == 0 ? tempty_leader0 : tempty_leader1);
      }
      if (row_ok && best_key != kKeyEmpty) {  // empty: every chunk fell below the row's best
        atomicMax(&args.keys[row], best_key);
        __threadfence();
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
  cluster_sync_all();  // the partner no longer touches this CTA's shared memory / TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }

  if (!STORE && args.idx_out != nullptr) {
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

}  // namespace dels
