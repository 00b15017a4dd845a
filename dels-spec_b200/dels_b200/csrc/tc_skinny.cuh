// Skinny draft scorer for decode-shaped calls (a few rows: the graph runners score one
// position of B sequences per step), sm_100a.
//
//   score[row, v] = (sum_k h[row, k] W[v, k]) + (sum_j s'[row, j] Vr[v, j])
//                   (+ base[row, v]) - beta_p * prior[v]          s' = alpha_p * s
//   token[row]    = argmax_v score[row, v]   (lowest index on ties)
//
// Same contraction and epilogue arithmetic as tc_gemm_kernel<kArgmax>, with the operand
// roles swapped: the vocab tile is the MMA's M side (128 TMEM lanes, one vocab row per
// epilogue thread) and the rows are its N side (NB = 16 or 32 columns).  Per K block
// a stage then holds 16 KB of the streamed weight and only NB x 128 B of rows, so eight
// stages keep ~150 KB of the weight in flight per SM, and every epilogue thread has
// work: it adds its vocab row's base logits and prior, packs (score, index) keys and
// keeps a running maximum per row in registers across all the tiles its CTA scores.
// With STAGE, the tile's base-logit rows and prior slice are fetched by the TMA producer
// into a per-accumulator shared-memory buffer a tile or more ahead (own full / empty
// barriers), so the epilogue never waits on global loads that queue behind the weight
// stream (at 16 rows that wait was ~3 us per tile); for a few rows the epilogue's own
// two loads per tile are cheaper than the extra hand-off, and it loads them directly.
// The maxima meet once per CTA (warp shuffles, then shared memory) before one 64-bit
// atomicMax per row.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue (TMEM lane quadrant = warp % 4); tc_skinny_gh_kernel adds warps
// 6..7, which compute the next rollout step's W_hh h while the others score.
// Reference: code/kernel/dels.py:49-79 + :443-456 (the per-step low-rank scorer and
// argmax of the greedy rollout) and code/dflash.py:468 (the long-logit GEMM).
#pragma once

#include "tc_gemm.cuh"

namespace dels {

constexpr int kSkinnyBM = 128;  // vocab rows per tile (MMA M)
constexpr int kSkinnyGhThreads = kTcThreads + 64;  // + two helper warps (tc_skinny_gh_kernel)
constexpr int kSkinnyGhMaxB = 4;                   // rows of the helpers' 4-row GEMV build
constexpr int kSkinnyGhRows = 8;                   // most rows of the scorer with helpers

// STAGE = false (the plain variant) leaves out the epilogue-operand buffers.  More stages
// for it (12 at NB = 16) measured slower in the batch-1 rollout.
template <int NB, bool STAGE = true>
struct SkinnyConfig {
  static_assert(NB == 16 || NB == 32, "NB is 16 or 32");
  static constexpr int kABytes = kSkinnyBM * kBK * 2;  // vocab tile: 128 x 64 bf16
  static constexpr int kBBytes = NB * kBK * 2;         // row tile: NB x 64 bf16
  static constexpr int kStages = 8;
  static constexpr int kAcc = 4;  // accumulators (tiles) in flight in TMEM
  static constexpr int kTmemCols = kAcc * NB <= 32 ? 32 : (kAcc * NB <= 64 ? 64 : 128);
  // per accumulator: the tile's base logits [NB][128] bf16 and prior [128] fp32
  static constexpr int kEpiBaseBytes = NB * kSkinnyBM * 2;
  static constexpr int kEpiPriorBytes = kSkinnyBM * 4;
  static constexpr int kEpiOffset = kStages * (kABytes + kBBytes);
  static constexpr int kBarOffset = kEpiOffset + (STAGE ? kAcc * (kEpiBaseBytes + kEpiPriorBytes) : 0);
  static constexpr int kNumBars = 2 * kStages + 4 * kAcc;
  static constexpr int kRedOffset = kBarOffset + kNumBars * 8 + 16;
  static constexpr int kSmemBytes = kRedOffset + 4 * NB * 8 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// `map_a0`/`map_a1`: the weights (W [V, H], Vr [V, r]) in 64 x 128 boxes; `map_b0`/`map_b1`:
// the rows (h [rows, H], alpha-scaled s [rows, r]) in 64 x NB boxes.  args.kb0 / kb1 are
// the K blocks of the two segments (kb0 = 0 for the base-logit variant).  With STAGE:
// `map_base` = base logits [rows, V slice] in 128 x NB boxes (when args.base is set) and
// `map_prior` = the prior [V slice] fp32 in 128-element boxes (when args.prior is set).
// GH: warps 6 and 7 compute args.gh_out (the next rollout step's W_hh h) for up to GHB
// rows, four output rows per warp at a time over a grid-wide stride, while warps 0-5
// score.  RB (<= NB) bounds
// the rows the epilogue scores at compile time: the MMA still computes NB columns, but a
// batch-1 step does not issue (predicated-off) epilogue arithmetic for the other 15.
template <int NB, bool STAGE, bool GH = false, int GHB = kSkinnyGhMaxB, int RB = NB>
__device__ __forceinline__ void skinny_body(const CUtensorMap* map_a0, const CUtensorMap* map_b0,
                                            const CUtensorMap* map_a1, const CUtensorMap* map_b1,
                                            const CUtensorMap* map_base, const CUtensorMap* map_prior,
                                            const TcArgs& args) {
  using Cfg = SkinnyConfig<NB, STAGE>;
  constexpr int S = Cfg::kStages;
  constexpr int NA = Cfg::kAcc;
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
  long long* red = reinterpret_cast<long long*>(smem + Cfg::kRedOffset);  // [4][NB]

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * S + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * S + NA + a]); };
  auto efull_bar = [&](int a) { return smem_u32(&bars[2 * S + 2 * NA + a]); };
  auto eempty_bar = [&](int a) { return smem_u32(&bars[2 * S + 3 * NA + a]); };
  auto epi_base = [&](int a) { return Cfg::kEpiOffset + a * (Cfg::kEpiBaseBytes + Cfg::kEpiPriorBytes); };
  const bool stage_base = STAGE && args.base != nullptr;
  const bool stage_prior = STAGE && args.prior != nullptr;
  const bool stage_epi = stage_base || stage_prior;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int num_tiles = (args.n_cols + kSkinnyBM - 1) / kSkinnyBM;
  const int total_kb = args.kb0 + args.kb1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < NA; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4 * 32);
      mbar_init(efull_bar(a), 1);
      mbar_init(eempty_bar(a), 4 * 32);
    }
    *abort_flag = 0;
    *last_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(map_a0);
    tma_prefetch_map(map_b0);
    tma_prefetch_map(map_a1);
    tma_prefetch_map(map_b1);
    if (stage_base) tma_prefetch_map(map_base);
    if (stage_prior) tma_prefetch_map(map_prior);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The weight tiles of the first S stages do not depend on any earlier kernel: in the
  // plain variant (a few rows) the producer issues them before the programmatic-
  // dependency wait, so in a rollout the weight stream starts while the previous step's
  // kernel finishes (batch-1 runner step -4 %).  Each prefetched stage already carries
  // its full expected byte count; its row-tile load follows after the wait.  The staged
  // variant does not prefetch: there the tile's epilogue operands would queue behind the
  // prefetched weights (measured +4 % at 16 rows).
  constexpr uint32_t tx = (uint32_t)(Cfg::kABytes + Cfg::kBBytes);
  const int my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int n_pre = STAGE ? 0 : min(S, my_tiles * total_kb);
  if (warp == 0 && lane == 0) {
    for (int it = 0; it < n_pre; ++it) {
      const int n0 = ((int)blockIdx.x + (it / total_kb) * (int)gridDim.x) * kSkinnyBM;
      const int kb = it % total_kb;
      mbar_arrive_expect_tx(full_bar(it), tx);
      if (kb < args.kb0)
        tma_load_2d(a_base + it * Cfg::kABytes, map_a0, full_bar(it), kb * kBK, n0);
      else
        tma_load_2d(a_base + it * Cfg::kABytes, map_a1, full_bar(it), (kb - args.kb0) * kBK, n0);
    }
  }
  // From here on the inputs of earlier kernels (rows, keys, device row count) are read.
  pdl_wait();
  int m_rows = args.m_rows;
  if (args.m_rows_dev != nullptr) {
    const int d = *args.m_rows_dev;
    m_rows = d < 0 ? 0 : (d < m_rows ? d : m_rows);
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      const uint32_t etx = (stage_base ? (uint32_t)Cfg::kEpiBaseBytes : 0u) +
                           (stage_prior ? (uint32_t)Cfg::kEpiPriorBytes : 0u);
      int eacc = 0, eissued = 0;
      uint32_t ephase = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int n0 = t * kSkinnyBM;
        if (stage_epi) {
          // the tile's epilogue operands, into the buffer of the accumulator it will use
          if (!mbar_wait(eempty_bar(eacc), ephase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(efull_bar(eacc), etx);
          const uint32_t eb = base_addr + (uint32_t)epi_base(eacc);
          if (stage_base) tma_load_2d(eb, map_base, efull_bar(eacc), n0, 0);
          if (stage_prior) tma_load_2d(eb + (uint32_t)Cfg::kEpiBaseBytes, map_prior, efull_bar(eacc), n0, 0);
          ++eissued;
          if (++eacc == NA) {
            eacc = 0;
            ephase ^= 1u;
          }
        }
        for (int kb = 0; kb < total_kb; ++kb) {
          const bool prefetched = issued < n_pre;  // weight tile already in flight
          if (!prefetched) {
            if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full_bar(stage), tx);
          }
          const uint32_t a_dst = a_base + stage * Cfg::kABytes;
          const uint32_t b_dst = b_base + stage * Cfg::kBBytes;
          if (kb < args.kb0) {
            if (!prefetched) tma_load_2d(a_dst, map_a0, full_bar(stage), kb * kBK, n0);
            tma_load_2d(b_dst, map_b0, full_bar(stage), kb * kBK, 0);
          } else {
            const int k1 = kb - args.kb0;
            if (!prefetched) tma_load_2d(a_dst, map_a1, full_bar(stage), k1 * kBK, n0);
            tma_load_2d(b_dst, map_b1, full_bar(stage), k1 * kBK, 0);
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
        const int eout = eissued < NA ? eissued : NA;
        int e = eacc;
        uint32_t ep = ephase;
        for (int i = 0; i < eout; ++i) {
          if (--e < 0) {
            e = NA - 1;
            ep ^= 1u;
          }
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(efull_bar(e), ep) && globaltimer_ns() - t0 < kWaitLimitNs / 20) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(kSkinnyBM, NB);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * NB);
        for (int kb = 0; kb < total_kb; ++kb) {
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
                        (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(stage));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit(tfull_bar(acc));
        if (++acc == NA) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok || *abort_flag) {
        // Drain: every MMA this thread issued completes before TMEM is released.
        const uint32_t drain = tfull_bar(acc);
        tc_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, acc_phase) && globaltimer_ns() - t0 < kWaitLimitNs / 20) {
        }
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp can access
    const int nrows = m_rows < RB ? m_rows : RB;
    float negb[RB];
#pragma unroll
    for (int b = 0; b < RB; ++b)
      negb[b] = (b < nrows && args.prior != nullptr) ? -__ldg(&args.beta[row_position(args.row_pos, b, args.n_pos)])
                                                     : 0.0f;
    long long run[RB];
#pragma unroll
    for (int b = 0; b < RB; ++b) run[b] = kKeyEmpty;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int vt = quad * 32 + lane;  // this thread's row within the tile
      const int v = t * kSkinnyBM + vt;  // ... and within the vocab slice
      const bool v_ok = v < args.n_cols;
      float bv[RB];
      float pv = 0.0f;
      if (!STAGE) {
        // loaded directly, before the accumulator wait so the latency overlaps the MMAs
        pv = (v_ok && args.prior != nullptr) ? __ldg(args.prior + v) : 0.0f;
#pragma unroll
        for (int b = 0; b < RB; ++b)
          bv[b] = (v_ok && args.base != nullptr && b < nrows)
                      ? __bfloat162float(args.base[(long long)b * args.ld_base + v])
                      : 0.0f;
      }
      if (stage_epi && !mbar_wait(efull_bar(acc), acc_phase, abort_flag, args.status)) break;
      const uint8_t* eb = smem + epi_base(acc);
      if (stage_base) {
        const __nv_bfloat16* bs = reinterpret_cast<const __nv_bfloat16*>(eb);
#pragma unroll
        for (int b = 0; b < RB; ++b) bv[b] = __bfloat162float(bs[b * kSkinnyBM + vt]);
      } else if (STAGE) {
#pragma unroll
        for (int b = 0; b < RB; ++b) bv[b] = 0.0f;
      }
      if (stage_prior) pv = reinterpret_cast<const float*>(eb + Cfg::kEpiBaseBytes)[vt];
      if (stage_epi) mbar_arrive(eempty_bar(acc));
      if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * NB);
      uint32_t d[NB];
      if constexpr (NB == 16) {
        tmem_ld_16cols(taddr, d);
      } else {
        tmem_ld_32cols(taddr, d);
      }
      tmem_ld_wait(d);
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
      if (v_ok) {
        const uint32_t vidx = (uint32_t)(args.v_begin + v);
#pragma unroll
        for (int b = 0; b < RB; ++b) {
          if (b < nrows) {
            float sc = __uint_as_float(d[b]) + bv[b];
            sc = fmaf(negb[b], pv, sc);
            const long long key = (long long)(((unsigned long long)(uint32_t)ordered_i32_dev(sc) << 32) |
                                              (unsigned long long)(0xFFFFFFFFu - vidx));
            run[b] = key > run[b] ? key : run[b];
          }
        }
      }
      if (++acc == NA) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Per row: maximum over the warp's lanes, then over the four epilogue warps.
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      if (b < nrows) {
        long long k = run[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const long long other = __shfl_xor_sync(0xFFFFFFFFu, k, o);
          k = other > k ? other : k;
        }
        if (lane == 0) red[quad * NB + b] = k;
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const int et = threadIdx.x - 64;  // 0..127 over the epilogue warps
    if (et < nrows && *abort_flag == 0) {
      long long k = red[et];
      for (int q = 1; q < 4; ++q) k = red[q * NB + et] > k ? red[q * NB + et] : k;
      if (k != kKeyEmpty) {
        atomicMax(&args.keys[et], k);
        // ordered before this CTA's completion count only when the last CTA decodes;
        // keys-only calls leave their visibility to the end of the grid
        if (args.idx_out != nullptr) __threadfence();
      }
    }
  } else if constexpr (GH) {
    // ---------------------------------------------------------------- helpers: gh_out
    // gh_x was written by an earlier kernel (complete after pdl_wait above); lanes stride
    // the row 16 bytes at a time, then a warp reduction per output row.
    if (args.gh_out != nullptr) {
      // A warp takes rows hw, hw + nhw, ... in groups of kRows; each lane loads its 16-byte
      // pieces of all the group's rows (up to 4 x 32 pieces per row per pass) before any
      // arithmetic, so a group costs one memory round trip instead of one per row.  The
      // row loop is compiled for GHB rows (predicated-off FMAs still take issue slots).
      constexpr int kRows = 4, kPieces = 4;
      const int nb = args.gh_b < GHB ? args.gh_b : GHB;
      const int k8n = args.gh_k / 8;
      const int hw = (int)blockIdx.x * 2 + (warp - 6);
      const int nhw = (int)gridDim.x * 2;
      for (int j0 = hw; j0 < args.gh_rows; j0 += nhw * kRows) {
        float acc[kRows][GHB];
#pragma unroll
        for (int g = 0; g < kRows; ++g)
#pragma unroll
          for (int b = 0; b < GHB; ++b) acc[g][b] = 0.0f;
        for (int c0 = 0; c0 < k8n; c0 += 32 * kPieces) {
          uint4 w[kRows][kPieces];
#pragma unroll
          for (int g = 0; g < kRows; ++g) {
            const int j = j0 + g * nhw;
#pragma unroll
            for (int q = 0; q < kPieces; ++q) {
              const int c = c0 + q * 32 + lane;
              w[g][q] = (j < args.gh_rows && c < k8n)
                            ? __ldg(reinterpret_cast<const uint4*>(args.gh_w + (long long)j * args.gh_k) + c)
                            : make_uint4(0u, 0u, 0u, 0u);
            }
          }
#pragma unroll
          for (int b = 0; b < GHB; ++b) {
            if (b < nb) {
#pragma unroll
              for (int q = 0; q < kPieces; ++q) {
                const int c = c0 + q * 32 + lane;
                const uint4 x = c < k8n ? reinterpret_cast<const uint4*>(args.gh_x + (long long)b * args.gh_k)[c]
                                        : make_uint4(0u, 0u, 0u, 0u);
                const float x0 = bf16_lo(x.x), x1 = bf16_hi(x.x), x2 = bf16_lo(x.y), x3 = bf16_hi(x.y);
                const float x4 = bf16_lo(x.z), x5 = bf16_hi(x.z), x6 = bf16_lo(x.w), x7 = bf16_hi(x.w);
#pragma unroll
                for (int g = 0; g < kRows; ++g) {
                  float a = acc[g][b];
                  a = fmaf(bf16_lo(w[g][q].x), x0, a);
                  a = fmaf(bf16_hi(w[g][q].x), x1, a);
                  a = fmaf(bf16_lo(w[g][q].y), x2, a);
                  a = fmaf(bf16_hi(w[g][q].y), x3, a);
                  a = fmaf(bf16_lo(w[g][q].z), x4, a);
                  a = fmaf(bf16_hi(w[g][q].z), x5, a);
                  a = fmaf(bf16_lo(w[g][q].w), x6, a);
                  a = fmaf(bf16_hi(w[g][q].w), x7, a);
                  acc[g][b] = a;
                }
              }
            }
          }
        }
#pragma unroll
        for (int g = 0; g < kRows; ++g) {
          const int j = j0 + g * nhw;
#pragma unroll
          for (int b = 0; b < GHB; ++b) {
            float a = acc[g][b];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
            if (lane == 0 && b < nb && j < args.gh_rows) {
              const float bj = args.gh_bias != nullptr ? __bfloat162float(args.gh_bias[j]) : 0.0f;
              args.gh_out[(long long)b * args.gh_rows + j] = __float2bfloat16_rn(a + bj);
            }
          }
        }
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

// Two entry points over the same body: the staged one takes the two epilogue-operand maps
// as well; the plain one keeps its parameter block at the four operand maps.
template <int NB, int RB = NB>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_skinny_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                     const __grid_constant__ CUtensorMap map_a1, const __grid_constant__ CUtensorMap map_b1,
                     const TcArgs args) {
  skinny_body<NB, false, false, kSkinnyGhMaxB, RB>(&map_a0, &map_b0, &map_a1, &map_b1, nullptr, nullptr, args);
}

// The plain scorer plus the helper warps that compute the next rollout step's gh, both for
// up to GHB rows.
template <int NB, int GHB>
__global__ void __launch_bounds__(kSkinnyGhThreads, 1)
    tc_skinny_gh_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                        const __grid_constant__ CUtensorMap map_a1, const __grid_constant__ CUtensorMap map_b1,
                        const TcArgs args) {
  skinny_body<NB, false, true, GHB, GHB>(&map_a0, &map_b0, &map_a1, &map_b1, nullptr, nullptr, args);
}

template <int NB>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_skinny_staged_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                            const __grid_constant__ CUtensorMap map_a1, const __grid_constant__ CUtensorMap map_b1,
                            const __grid_constant__ CUtensorMap map_base, const __grid_constant__ CUtensorMap map_prior,
                            const TcArgs args) {
  skinny_body<NB, true>(&map_a0, &map_b0, &map_a1, &map_b1, &map_base, &map_prior, args);
}

}  // namespace dels
