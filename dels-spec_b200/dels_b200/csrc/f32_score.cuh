// Declarations for the fp32 (CUDA-core) draft scorer; see f32_score.cu.
#pragma once

#include "common.cuh"

namespace dels {

constexpr int kF32Threads = 288;  // 8 compute warps + 1 TMA producer warp


__global__ void f32_rank_kernel(const float* __restrict__ h, long long ld_h, const float* __restrict__ ut,
                                long long ld_ut, int rows, int H, int r, const float* __restrict__ alpha,
                                int n_pos, const int* __restrict__ row_pos, float* s_scaled, long long* keys,
                                unsigned* counter);

__global__ void f32_transpose_pass_kernel(const float* __restrict__ h, long long ld_h, int H,
                                          const float* __restrict__ s, long long ld_s, int r, int nrows,
                                          float* __restrict__ hT, float* __restrict__ sT);

// Sets the dynamic shared-memory limit of the fp32 scorer and loads it.
cudaError_t f32_score_setup(int max_smem);
int f32_score_smem_bytes();
// Vocabulary rows per tile of the fp32 scorer (the box height of its W / Vr tensor maps).
int f32_score_tile_rows();

// One pass of the fp32 scorer over data rows [row0, row0 + nrows), nrows <= 16.
// map_w / map_vr: fp32 [V, H] / [V, r], box 32 x f32_score_tile_rows() rows, 128-byte swizzle;
// map_h / map_s: the pass's rows transposed, fp32 [H][16] / [r][16], box 16 x 32 k, no
// swizzle (f32_transpose_pass_kernel).
cudaError_t f32_score_launch(int grid, cudaStream_t st, const CUtensorMap& map_w, const CUtensorMap& map_h,
                             const CUtensorMap& map_vr, const CUtensorMap& map_s, int kb0, int kb1,
                             const float* prior, const float* beta, int n_pos, const int* row_pos, int row0,
                             int nrows, int V, long long v_begin, long long* keys, int* status);

}  // namespace dels
