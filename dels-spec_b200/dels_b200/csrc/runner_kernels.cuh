// Declarations of the small-batch rollout kernels (definitions in runner_kernels.cu).
#pragma once

#include "common.cuh"

namespace dels {

constexpr int kRunnerMaxB = 16;  // rows staged in shared memory per pass
constexpr int kGruCols = 4;      // hidden units per CTA in the GRU step
constexpr int kGruThreads = 3 * kGruCols * 32;  // one warp per gate row of the CTA's units
constexpr int kGemvThreads = 128;

inline size_t gru_smem_bytes(int G) {
  return (size_t)kRunnerMaxB * G * 2 + (size_t)3 * kGruCols * kRunnerMaxB * 4;
}
inline size_t rank_gemv_smem_bytes(int K) { return (size_t)kRunnerMaxB * K * 2; }

__global__ void gru_step_kernel(const long long* __restrict__ tokens, long long tok_stride,
                                const __nv_bfloat16* __restrict__ table, long long ld_table,
                                const __nv_bfloat16* __restrict__ w_hh, const __nv_bfloat16* __restrict__ b_hh,
                                const __nv_bfloat16* h_in, __nv_bfloat16* h_out, int B, int G, int V, int* status);

__global__ void rank_gemv_kernel(const __nv_bfloat16* __restrict__ x, long long ld_x,
                                 const __nv_bfloat16* __restrict__ w, long long ld_w,
                                 const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ addend,
                                 long long ld_add, int B, int K, int r, int activation,
                                 const float* __restrict__ alpha, int n_pos, const int* __restrict__ row_pos,
                                 __nv_bfloat16* s_out, __nv_bfloat16* s_scaled, long long* keys, unsigned* counter);

__global__ void gru_gates_kernel(const long long* __restrict__ tokens, long long tok_stride,
                                 const __nv_bfloat16* __restrict__ table, long long ld_table,
                                 const __nv_bfloat16* __restrict__ gh, long long ld_gh, const __nv_bfloat16* h_in,
                                 __nv_bfloat16* h_out, int B, int G, int V, int* status);

__global__ void gather_scaled_kernel(const long long* __restrict__ tokens, long long tok_stride,
                                     const __nv_bfloat16* __restrict__ emb, long long ld_emb,
                                     const float* __restrict__ alpha, int n_pos, int B, int r, int V,
                                     __nv_bfloat16* s_scaled, long long* keys, unsigned* counter, int* status);

}  // namespace dels
