// fp32 draft scorer on the CUDA cores (fp32 workloads with a 1e-5 score tolerance, so the
// contraction stays in IEEE fp32 FMAs; TF32 tensor cores would not meet it).
//
//   s'[row, j]     = alpha_p * sum_k h[row, k] * U^T[j, k]                 (prologue)
//   score[row, v]  = sum_k W[v, k] h[row, k] + sum_j Vr[v, j] s'[row, j] - beta_p * prior[v]
//   token[row]     = argmax_v score[row, v]   (lowest index on ties)
//
// Reference formula: code/kernel/dels.py:447-456 (torch fallback) with the long
// logits of code/dflash.py:468 fused in and the rank state of code/dels.py:334-339.
//
// The scorer is an HBM-bound multi-row GEMV: every W element is read once and used
// for all rows of the pass.  Each warp streams NV=8 vocabulary rows of [W | Vr] with
// coalesced 16-byte loads (lane l owns k = 4l..4l+3 of every 128-wide chunk), keeps
// ROWS x NV partial dot products in registers, and reads the rows' [h | s'] from
// shared memory.  A 5-stage recursive-halving shuffle then reduce-scatters the
// partials so each lane ends with complete scores for one row, applies the prior, and
// keeps a running packed (score, index) key; one 64-bit atomicMax per (row, warp)
// merges the warps.
#include "f32_score.cuh"

namespace dels {

// Register select that the compiler cannot turn into an indexed (local-memory) access
// of the partial-sum array.
__device__ __forceinline__ float select_f32(bool c, float a, float b) {
  float r;
  asm("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\tselp.f32 %0, %1, %2, p;\n\t}"
      : "=f"(r)
      : "f"(a), "f"(b), "r"((int)c));
  return r;
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

template <int ROWS>
__global__ void __launch_bounds__(kF32Threads, 1)
    f32_score_kernel(const float* __restrict__ h, long long ld_h, const float* __restrict__ s_scaled,
                     const float* __restrict__ W, long long ld_w, const float* __restrict__ vr, long long ld_vr,
                     const float* __restrict__ prior, const float* __restrict__ beta, int n_pos,
                     const int* __restrict__ row_pos, int row0, int nrows, int H, int r, int V, long long v_begin,
                     long long* keys) {
  constexpr int NV = ROWS >= 16 ? 4 : 8;  // vocabulary rows per warp iteration
  constexpr int N = ROWS * NV;  // partial sums per lane
  constexpr int PER_LANE = N / 32;
  constexpr int LANES_PER_ROW = NV / PER_LANE;
  static_assert(N >= 32 && (N % 32) == 0, "ROWS * NV must be a multiple of 32");
  extern __shared__ float4 a_s4[];
  float* a_s = reinterpret_cast<float*>(a_s4);

  const int kp = f32_padded_k(H, r);  // padded K' = H + r rounded up to 128
  // Stage [h | s' | 0] for the pass's rows in shared memory.
  for (int e = threadIdx.x; e < ROWS * kp; e += blockDim.x) {
    const int rr = e / kp, k = e % kp;
    float x = 0.0f;
    if (rr < nrows) {
      if (k < H)
        x = h[(long long)(row0 + rr) * ld_h + k];
      else if (k - H < r)
        x = s_scaled[(long long)(row0 + rr) * r + (k - H)];
    }
    a_s[e] = x;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gwarp = blockIdx.x * (kF32Threads / 32) + warp;
  const int nwarps = gridDim.x * (kF32Threads / 32);
  const int ngroups = (V + NV - 1) / NV;
  const int nchunks = kp / 128;

  const int my_row = (lane * PER_LANE) / NV;
  const int my_vi0 = (lane * PER_LANE) % NV;
  float negb = 0.0f;
  if (my_row < nrows && prior != nullptr) negb = -beta[row_position(row_pos, row0 + my_row, n_pos)];
  long long best_key = kKeyEmpty;

  for (int g = gwarp; g < ngroups; g += nwarps) {
    const int v0 = g * NV;
    float acc[N];
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = 0.0f;

#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
      const int k = c * 128 + 4 * lane;
      float4 w[NV];
#pragma unroll
      for (int vi = 0; vi < NV; ++vi) {
        const int v = v0 + vi;
        w[vi] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (v < V) {
          if (k < H)
            w[vi] = __ldg(reinterpret_cast<const float4*>(W + (long long)v * ld_w + k));
          else if (k - H < r)
            w[vi] = __ldg(reinterpret_cast<const float4*>(vr + (long long)v * ld_vr + (k - H)));
        }
      }
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr) {
        const float4 a = a_s4[(rr * kp + k) >> 2];
#pragma unroll
        for (int vi = 0; vi < NV; ++vi) {
          float t = acc[rr * NV + vi];
          t = fmaf(a.x, w[vi].x, t);
          t = fmaf(a.y, w[vi].y, t);
          t = fmaf(a.z, w[vi].z, t);
          t = fmaf(a.w, w[vi].w, t);
          acc[rr * NV + vi] = t;
        }
      }
    }

    // Recursive-halving reduce-scatter: afterwards lane l holds the complete sums of
    // partial-index l*PER_LANE + j, j < PER_LANE (index = row * NV + vi).
#pragma unroll
    for (int st = 0; st < 5; ++st) {
      const int o = 16 >> st;
      const int half = N >> (st + 1);
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < half; ++j) {
        const float lo = acc[j], hi = acc[j + half];
        const float send = select_f32(upper, lo, hi);
        const float keep = select_f32(upper, hi, lo);
        acc[j] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
      }
    }

    if (my_row < nrows) {
#pragma unroll
      for (int j = 0; j < PER_LANE; ++j) {
        const int v = v0 + my_vi0 + j;
        if (v < V) {
          float s = acc[j];
          if (prior != nullptr) s = fmaf(negb, __ldg(prior + v), s);
          const long long key = pack_key(s, (uint32_t)(v_begin + v));
          best_key = key > best_key ? key : best_key;
        }
      }
    }
  }

  // Lanes that share a row combine, then one atomic per (row, warp).
#pragma unroll
  for (int o = 1; o < LANES_PER_ROW; o <<= 1) {
    const long long other = __shfl_xor_sync(0xFFFFFFFFu, best_key, o);
    best_key = other > best_key ? other : best_key;
  }
  if ((lane % LANES_PER_ROW) == 0 && my_row < nrows && best_key != kKeyEmpty)
    atomicMax(&keys[row0 + my_row], best_key);
}

cudaError_t f32_score_setup(int max_smem) {
  cudaError_t e;
  cudaFuncAttributes attr;
  if ((e = cudaFuncSetAttribute(f32_score_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(f32_score_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(f32_score_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess) return e;
  if ((e = cudaFuncGetAttributes(&attr, f32_score_kernel<16>)) != cudaSuccess) return e;
  if ((e = cudaFuncGetAttributes(&attr, f32_score_kernel<8>)) != cudaSuccess) return e;
  return cudaFuncGetAttributes(&attr, f32_score_kernel<4>);
}

cudaError_t f32_score_launch(int rows_per_pass, int grid, size_t smem, cudaStream_t st, const float* h, long long ld_h,
                             const float* s_scaled, const float* W, long long ld_w, const float* vr, long long ld_vr,
                             const float* prior, const float* beta, int n_pos, const int* row_pos, int row0,
                             int nrows, int H, int r, int V, long long v_begin, long long* keys) {
  switch (rows_per_pass) {
    case 16:
      f32_score_kernel<16><<<grid, kF32Threads, smem, st>>>(h, ld_h, s_scaled, W, ld_w, vr, ld_vr, prior, beta, n_pos,
                                                            row_pos, row0, nrows, H, r, V, v_begin, keys);
      break;
    case 8:
      f32_score_kernel<8><<<grid, kF32Threads, smem, st>>>(h, ld_h, s_scaled, W, ld_w, vr, ld_vr, prior, beta, n_pos,
                                                           row_pos, row0, nrows, H, r, V, v_begin, keys);
      break;
    default:
      f32_score_kernel<4><<<grid, kF32Threads, smem, st>>>(h, ld_h, s_scaled, W, ld_w, vr, ld_vr, prior, beta, n_pos,
                                                           row_pos, row0, nrows, H, r, V, v_begin, keys);
      break;
  }
  return cudaGetLastError();
}

}  // namespace dels
