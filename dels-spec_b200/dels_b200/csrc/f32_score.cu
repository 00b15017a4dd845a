// fp32 draft scorer on the CUDA cores (fp32 workloads with a 1e-5 score tolerance, so the
// contraction stays in IEEE fp32 FMAs: a split-TF32 tensor-core variant measured 1.2e-5
// worst-case error and ran slower at 16 rows).
//
//   s'[row, j]     = alpha_p * sum_k h[row, k] * U^T[j, k]                 (prologue)
//   score[row, v]  = sum_k W[v, k] h[row, k] + sum_j Vr[v, j] s'[row, j] - beta_p * prior[v]
//   token[row]     = argmax_v score[row, v]   (lowest index on ties)
//
// Reference formula: code/kernel/dels.py:447-456 (torch fallback) with the long
// logits of code/dflash.py:468 fused in and the rank state of code/dels.py:334-339.
//
// The scorer is an HBM-bound multi-row GEMV: every W element is read once and used
// for all 16 rows of a pass.  The design is described above f32_score_kernel.
#include "f32_score.cuh"

namespace dels {

// The data rows of one pass, transposed: dst[k][16] = src[r][k] for r < nrows, zero for
// the padding rows, for both segments (h over H, s' over r) in one launch.  The scorer
// then reads one k of all 16 rows as four 16-byte shared-memory broadcasts.
__global__ void f32_transpose_pass_kernel(const float* __restrict__ h, long long ld_h, int H,
                                          const float* __restrict__ s, long long ld_s, int r, int nrows,
                                          float* __restrict__ hT, float* __restrict__ sT) {
  const long long nh = (long long)H * 16, total = nh + (long long)r * 16;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const bool seg0 = e < nh;
    const long long f = seg0 ? e : e - nh;
    const int k = (int)(f >> 4), row = (int)(f & 15);
    float v = 0.0f;
    if (row < nrows) v = seg0 ? h[row * ld_h + k] : s[row * ld_s + k];
    (seg0 ? hT : sT)[f] = v;
  }
}

__global__ void f32_rank_kernel(const float* __restrict__ h, long long ld_h, const float* __restrict__ ut,
                                long long ld_ut, int rows, int H, int r, const float* __restrict__ alpha,
                                int n_pos, const int* __restrict__ row_pos, float* s_scaled, long long* keys,
                                unsigned* counter) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int o = warp; o < rows * r; o += nwarps) {
    const int row = o / r, j = o % r;
    const float* hr = h + (long long)row * ld_h;
    const float* ur = ut + (long long)j * ld_ut;
    float acc = 0.0f;
    for (int k = lane; k < H; k += 32) acc = fmaf(hr[k], ur[k], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
    if (lane == 0) {
      const float a = alpha != nullptr ? alpha[row_position(row_pos, row, n_pos)] : 1.0f;
      s_scaled[o] = a * acc;
      if (j == 0 && keys != nullptr) keys[row] = kKeyEmpty;
    }
  }
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
}

// ------------------------------------------------------------------------------------
// fp32 scorer.  Persistent: CTA c owns a contiguous run of 96-token vocabulary tiles
// (1583 tiles at V = 151936: at most 11 per CTA on 148 SMs, 3 % above an even split).
// Each K block of 64 is staged by TMA: the tile's 96 W rows (two 32-float boxes, 128-byte
// swizzle, so the 32 rows a warp reads at one k fall in 8 distinct 16-byte bank groups)
// and the pass's 16 data rows transposed ([k][16], two boxes of 32 k, read as
// shared-memory broadcasts).  Compute warp w owns the 8-wide K slice made of 16-byte
// chunks 2(w % 4) and 2(w % 4) + 1 of box w / 4, and keeps, per lane, 3 vocabulary rows
// (lane + 32 j) x 16 data rows of partial sums in registers as pairs of data rows: one
// packed two-lane FMA (__ffma2_rn, the rounding of two fmaf) updates two data rows.  One
// 16-byte broadcast of the data rows thus feeds 3 x 2 packed FMAs per lane; with two
// vocabulary rows per lane (64-row tiles) the broadcasts made the shared-memory pipe
// the busiest unit (75 % of peak, ncu) and serialised with the FP32 pipe.  After the
// last K block the 8 slices are summed through shared memory ([warp][row quad][v],
// conflict-free), the prior term applied, and each thread keeps running packed (score,
// index) keys for 8 data rows of one vocabulary row.  A ninth warp issues the TMA loads
// (6-stage mbarrier ring, bounded waits).
// ------------------------------------------------------------------------------------
namespace {
constexpr int kF32TileV = 96;                       // vocabulary rows per tile (3 per lane)
constexpr int kF32VPerLane = kF32TileV / 32;
constexpr int kF32Rows = 16;                        // data rows per pass
constexpr int kF32KB = 64;                          // K per stage
constexpr int kF32WBox = 32 * kF32TileV * 4;        // one 32-float x 96-row box: 12 KB
constexpr int kF32HBox = 32 * kF32Rows * 4;         // one 32-float x 16-row box: 2 KB
constexpr int kF32StageBytes = 2 * kF32WBox + 2 * kF32HBox;  // 28 KB
constexpr int kF32Stages = 6;
constexpr int kF32ComputeWarps = kF32Threads / 32 - 1;       // 8
constexpr int kF32EpiThreads = 2 * kF32TileV;                // (vocabulary row, 8 data rows)
constexpr int kF32RedBytes = kF32ComputeWarps * kF32TileV * kF32Rows * 4;  // 48 KB
static_assert(kF32ComputeWarps == 8, "8 compute warps x 8-wide K slices cover a 64-wide K block");
static_assert(kF32EpiThreads <= kF32ComputeWarps * 32, "epilogue threads");
}  // namespace

int f32_score_smem_bytes() { return kF32Stages * kF32StageBytes + kF32RedBytes + 256 + 1024; }
int f32_score_tile_rows() { return kF32TileV; }

__global__ void __launch_bounds__(kF32Threads, 1)
    f32_score_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_h,
                     const __grid_constant__ CUtensorMap map_vr, const __grid_constant__ CUtensorMap map_s,
                     int kb0, int kb1, const float* __restrict__ prior, const float* __restrict__ beta, int n_pos,
                     const int* __restrict__ row_pos, int row0, int nrows, int V, long long v_begin,
                     long long* keys, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);
  float* red = reinterpret_cast<float*>(smem + kF32Stages * kF32StageBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kF32Stages * kF32StageBytes + kF32RedBytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kF32Stages);
  auto full_bar = [&](int st) { return smem_u32(&bars[st]); };
  auto empty_bar = [&](int st) { return smem_u32(&bars[kF32Stages + st]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (V + kF32TileV - 1) / kF32TileV;
  const int t_lo = (int)((long long)tiles * blockIdx.x / gridDim.x);
  const int t_hi = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
  const int nkb = kb0 + kb1;

  if (threadIdx.x == 0) {
    for (int st = 0; st < kF32Stages; ++st) {
      mbar_init(full_bar(st), 1);
      mbar_init(empty_bar(st), kF32ComputeWarps);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kF32ComputeWarps) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int st = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = t_lo; t < t_hi && ok; ++t) {
        const int v0 = t * kF32TileV;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(empty_bar(st), phase ^ 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          const uint32_t dst = base_addr + st * kF32StageBytes;
          mbar_arrive_expect_tx(full_bar(st), kF32StageBytes);
          const bool seg0 = kb < kb0;
          const int k = (seg0 ? kb : kb - kb0) * kF32KB;
          const CUtensorMap* mw = seg0 ? &map_w : &map_vr;
          const CUtensorMap* mh = seg0 ? &map_h : &map_s;
          tma_load_2d(dst, mw, full_bar(st), k, v0);
          tma_load_2d(dst + kF32WBox, mw, full_bar(st), k + 32, v0);
          tma_load_2d(dst + 2 * kF32WBox, mh, full_bar(st), 0, k);
          tma_load_2d(dst + 2 * kF32WBox + kF32HBox, mh, full_bar(st), 0, k + 32);
          if (++st == kF32Stages) {
            st = 0;
            phase ^= 1u;
          }
        }
      }
    }
    return;  // the producer takes no part in the reduction barriers below
  }

  // -------------------------------------------------------------- compute warps
  const int box = warp >> 2;            // which 32-wide half of the K block
  const int cp = (warp & 3) * 2;        // this warp's first 16-byte chunk of each 128-byte row
  // epilogue ownership: vocabulary row v_e of the tile, data rows [8 rq, 8 rq + 8)
  const bool epi = threadIdx.x < kF32EpiThreads;
  const int v_e = threadIdx.x % kF32TileV;
  const int rq = threadIdx.x / kF32TileV;
  float negb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 8 * rq + i;
    negb[i] = (epi && r < nrows && prior != nullptr) ? -beta[row_position(row_pos, row0 + r, n_pos)] : 0.0f;
  }
  long long best[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) best[i] = kKeyEmpty;
  int st = 0;
  uint32_t phase = 0;
  bool ok = true;
  float4* red4 = reinterpret_cast<float4*>(red);  // [warp][row quad][v]

  for (int t = t_lo; t < t_hi && ok; ++t) {
    const int v0 = t * kF32TileV;
    float2 acc[kF32VPerLane][kF32Rows / 2];  // acc[j][p] = partial sums of data rows (2p, 2p + 1)
#pragma unroll
    for (int j = 0; j < kF32VPerLane; ++j)
#pragma unroll
      for (int p = 0; p < kF32Rows / 2; ++p) acc[j][p] = make_float2(0.0f, 0.0f);

    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(full_bar(st), phase, abort_flag, status)) {
        ok = false;
        break;
      }
      const uint8_t* stage = smem + st * kF32StageBytes;
      const uint8_t* wbox = stage + box * kF32WBox;
      const float* hbox = reinterpret_cast<const float*>(stage + 2 * kF32WBox + box * kF32HBox);  // [32 k][16]
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = cp + cc;
        float4 w[kF32VPerLane];
#pragma unroll
        for (int j = 0; j < kF32VPerLane; ++j) {
          const int v = lane + 32 * j;
          w[j] = *reinterpret_cast<const float4*>(wbox + v * 128 + ((c ^ (v & 7)) << 4));
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const float4* hk = reinterpret_cast<const float4*>(hbox + (c * 4 + kk) * kF32Rows);
          float4 hv[kF32Rows / 4];
#pragma unroll
          for (int q = 0; q < kF32Rows / 4; ++q) hv[q] = hk[q];  // data rows 4q .. 4q+3 at this k
#pragma unroll
          for (int j = 0; j < kF32VPerLane; ++j) {
            const float wk = kk == 0 ? w[j].x : (kk == 1 ? w[j].y : (kk == 2 ? w[j].z : w[j].w));
            const float2 w2 = make_float2(wk, wk);
#pragma unroll
            for (int q = 0; q < kF32Rows / 4; ++q) {
              acc[j][2 * q] = __ffma2_rn(w2, make_float2(hv[q].x, hv[q].y), acc[j][2 * q]);
              acc[j][2 * q + 1] = __ffma2_rn(w2, make_float2(hv[q].z, hv[q].w), acc[j][2 * q + 1]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(st));
      if (++st == kF32Stages) {
        st = 0;
        phase ^= 1u;
      }
    }
    if (!ok) break;

    // sum the 8 K slices: red4[warp][q][v] holds data rows 4q .. 4q+3 of vocabulary row v
#pragma unroll
    for (int j = 0; j < kF32VPerLane; ++j)
#pragma unroll
      for (int q = 0; q < kF32Rows / 4; ++q)
        red4[(warp * 4 + q) * kF32TileV + lane + 32 * j] =
            make_float4(acc[j][2 * q].x, acc[j][2 * q].y, acc[j][2 * q + 1].x, acc[j][2 * q + 1].y);
    asm volatile("bar.sync 1, %0;" ::"r"(kF32ComputeWarps * 32) : "memory");
    if (epi && v0 + v_e < V) {
      float sum[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] = 0.0f;
#pragma unroll
      for (int w8 = 0; w8 < kF32ComputeWarps; ++w8) {
        const float4 a = red4[(w8 * 4 + 2 * rq) * kF32TileV + v_e];
        const float4 b = red4[(w8 * 4 + 2 * rq + 1) * kF32TileV + v_e];
        sum[0] += a.x;
        sum[1] += a.y;
        sum[2] += a.z;
        sum[3] += a.w;
        sum[4] += b.x;
        sum[5] += b.y;
        sum[6] += b.z;
        sum[7] += b.w;
      }
      const float pv = prior != nullptr ? __ldg(prior + v0 + v_e) : 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (8 * rq + i < nrows) {
          const float sc = prior != nullptr ? fmaf(negb[i], pv, sum[i]) : sum[i];
          const long long key = pack_key(sc, (uint32_t)(v_begin + v0 + v_e));
          best[i] = key > best[i] ? key : best[i];
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kF32ComputeWarps * 32) : "memory");
  }

  if (!ok) {
    // Aborted: give the producer's copies in flight time to land before leaving.
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < kWaitLimitNs / 40) {
    }
  }
  // Per data row: maximum over the lanes of each warp (a warp's lanes share rq), then
  // over the three warps that own the row, one atomic per (row, CTA).
  long long* rb = reinterpret_cast<long long*>(red);  // [warp][8], the sums are no longer needed
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    long long k = best[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long other = __shfl_xor_sync(0xFFFFFFFFu, k, o);
      k = other > k ? other : k;
    }
    best[i] = k;
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) rb[warp * 8 + i] = epi ? best[i] : kKeyEmpty;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kF32ComputeWarps * 32) : "memory");
  if (threadIdx.x < kF32Rows && (int)threadIdx.x < nrows) {
    const int r = threadIdx.x, q = r >> 3, i = r & 7;
    constexpr int kWarpsPerQ = kF32TileV / 32;
    long long k = kKeyEmpty;
    for (int w8 = q * kWarpsPerQ; w8 < (q + 1) * kWarpsPerQ; ++w8) k = rb[w8 * 8 + i] > k ? rb[w8 * 8 + i] : k;
    if (k != kKeyEmpty) atomicMax(&keys[row0 + r], k);
  }
}

cudaError_t f32_score_setup(int /*max_smem*/) {
  cudaError_t e = cudaFuncSetAttribute(f32_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       f32_score_smem_bytes());
  if (e != cudaSuccess) return e;
  cudaFuncAttributes attr;
  return cudaFuncGetAttributes(&attr, f32_score_kernel);
}

cudaError_t f32_score_launch(int grid, cudaStream_t st, const CUtensorMap& map_w, const CUtensorMap& map_h,
                             const CUtensorMap& map_vr, const CUtensorMap& map_s, int kb0, int kb1,
                             const float* prior, const float* beta, int n_pos, const int* row_pos, int row0,
                             int nrows, int V, long long v_begin, long long* keys, int* status) {
  f32_score_kernel<<<grid, kF32Threads, f32_score_smem_bytes(), st>>>(map_w, map_h, map_vr, map_s, kb0, kb1, prior,
                                                                      beta, n_pos, row_pos, row0, nrows, V, v_begin,
                                                                      keys, status);
  return cudaGetLastError();
}

}  // namespace dels
