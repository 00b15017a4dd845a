// Declarations of the small-batch rollout kernels (definitions in runner_kernels.cu).
#pragma once

#include "common.cuh"

namespace dels {

constexpr int kRunnerMaxB = 16;  // most rows staged in shared memory per pass
constexpr int kGruCols = 4;      // hidden units per CTA in the GRU step
constexpr int kGruThreads = 3 * kGruCols * 32;  // one warp per gate row of the CTA's units
constexpr int kGemvThreads = 128;

// rows per pass for a batch of B rows: the smallest of 1, 2, 4, 8, kRunnerMaxB holding B
inline int runner_rows_per_pass(int B) {
  return B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : kRunnerMaxB;
}
inline size_t gru_smem_bytes(int G, int rows_per_pass = kRunnerMaxB) {
  return (size_t)rows_per_pass * G * 2 + (size_t)3 * kGruCols * rows_per_pass * 4;
}
inline size_t rank_gemv_smem_bytes(int K, int rows_per_pass = kRunnerMaxB) {
  return (size_t)rows_per_pass * K * 2;
}

// x of rank_gemv_kernel computed in place as the GRU's new hidden state (table == null:
// x is read from memory): h_out[b] = GRU gates of (gi = table[tokens[b * tok_stride]],
// gh[b], h_in[b]), staged in shared memory by every CTA and stored by CTA 0.
struct GruGateSrc {
  const long long* tokens;     // token ids, or (token_keys) the previous step's packed argmax keys
  long long tok_stride;
  int token_keys;
  const __nv_bfloat16* table;  // [V, 3G] input projections, or null
  long long ld_table;
  const __nv_bfloat16* gh;     // [B, 3G] bf16(W_hh h + b_hh)
  long long ld_gh;
  const __nv_bfloat16* h_in;   // [B, G], null = zero state
  __nv_bfloat16* h_out;        // [B, G]
  int V;
  int* status;
};

// One GRU unit (code/kernel/dels.py:368-373): r, z = sigmoid(gi + gh), n = tanh(gi_n + r gh_n),
// h' = (1 - z) n + z h, in fp32 with the products pinned to explicit FMAs so that every
// kernel that evaluates it rounds alike.
__device__ __forceinline__ float sigmoid_unit(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float gru_unit(float gi_r, float gi_z, float gi_n, float gh_r, float gh_z, float gh_n,
                                          float h) {
  const float rg = sigmoid_unit(gi_r + gh_r);
  const float zg = sigmoid_unit(gi_z + gh_z);
  const float ng = tanhf(fmaf(rg, gh_n, gi_n));
  return fmaf(zg, h, (1.0f - zg) * ng);
}

// gru_step_kernel and rank_gemv_kernel, compiled for 1, 2, 4, 8 or kRunnerMaxB rows per
// pass (pick with runner_rows_per_pass; other values give the kRunnerMaxB build).
using GruStepKernel = void (*)(const long long* tokens, long long tok_stride, int token_keys, const __nv_bfloat16* table,
                               long long ld_table, const __nv_bfloat16* w_hh, const __nv_bfloat16* b_hh,
                               const __nv_bfloat16* h_in, __nv_bfloat16* h_out, int B, int G, int V, int* status);
using RankGemvKernel = void (*)(const __nv_bfloat16* x, long long ld_x, const __nv_bfloat16* w, long long ld_w,
                                const __nv_bfloat16* bias, const __nv_bfloat16* addend, long long ld_add, int B,
                                int K, int r, int activation, const float* alpha, int n_pos, const int* row_pos,
                                __nv_bfloat16* s_out, __nv_bfloat16* s_scaled, long long* keys, unsigned* counter,
                                const GruGateSrc gate);
GruStepKernel gru_step_kernel_for(int rows_per_pass);
RankGemvKernel rank_gemv_kernel_for(int rows_per_pass);

__global__ void gru_gates_kernel(const long long* __restrict__ tokens, long long tok_stride, int token_keys,
                                 const __nv_bfloat16* __restrict__ table, long long ld_table,
                                 const __nv_bfloat16* __restrict__ gh, long long ld_gh, const __nv_bfloat16* h_in,
                                 __nv_bfloat16* h_out, int B, int G, int V, int* status);

__global__ void gru_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                    long long ld_part, const long long* __restrict__ tokens, long long tok_stride,
                                    int token_keys, const __nv_bfloat16* __restrict__ table, long long ld_table,
                                    const __nv_bfloat16* __restrict__ b_hh, const __nv_bfloat16* h_in,
                                    __nv_bfloat16* h_out, int B, int G, int V, int* status);

__global__ void gather_scaled_kernel(const long long* __restrict__ tokens, long long tok_stride, int token_keys,
                                     const __nv_bfloat16* __restrict__ emb, long long ld_emb,
                                     const float* __restrict__ alpha, int n_pos, int B, int r, int V,
                                     __nv_bfloat16* s_scaled, long long* keys, unsigned* counter, int* status);

}  // namespace dels
