// Declarations for the fp32 (CUDA-core) draft scorer; see f32_score.cu.
#pragma once

#include "common.cuh"

namespace dels {

constexpr int kF32Threads = 256;

__host__ __device__ inline int f32_padded_k(int H, int r) { return ((H + r + 127) / 128) * 128; }

__global__ void f32_rank_kernel(const float* __restrict__ h, long long ld_h, const float* __restrict__ ut,
                                long long ld_ut, int rows, int H, int r, const float* __restrict__ alpha,
                                int n_pos, const int* __restrict__ row_pos, float* s_scaled, long long* keys,
                                unsigned* counter);

// Sets the dynamic shared-memory limit of every fp32 scorer specialisation and loads them.
cudaError_t f32_score_setup(int max_smem);

// One pass of the fp32 scorer over rows [row0, row0 + nrows); rows_per_pass is 16, 8 or 4.
cudaError_t f32_score_launch(int rows_per_pass, int grid, size_t smem, cudaStream_t st, const float* h, long long ld_h,
                             const float* s_scaled, const float* W, long long ld_w, const float* vr, long long ld_vr,
                             const float* prior, const float* beta, int n_pos, const int* row_pos, int row0,
                             int nrows, int H, int r, int V, long long v_begin, long long* keys);

}  // namespace dels
