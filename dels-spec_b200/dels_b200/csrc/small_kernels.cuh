// Declarations of the SIMT helper kernels (definitions in small_kernels.cu).
#pragma once

#include "common.cuh"

namespace dels {

constexpr int kRnnSeqs = 4;  // sequences per CTA in the RNN recurrence

__global__ void rank_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                     long long ld_part, int rows, int r, int activation, const float* __restrict__ alpha,
                                     int n_pos, const int* __restrict__ row_pos, __nv_bfloat16* s_out,
                                     __nv_bfloat16* s_scaled, long long* keys, unsigned* counter);

__global__ void correction_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                           long long ld_part, int rows, int m, const __nv_bfloat16* __restrict__ z,
                                           long long ld_z, const float* __restrict__ alpha, __nv_bfloat16* s_scaled,
                                           long long* keys, unsigned* counter);
__global__ void linear_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                       long long ld_part, int rows, int n, const __nv_bfloat16* __restrict__ bias,
                                       __nv_bfloat16* out, long long ld_out);

__global__ void keys_init_kernel(long long* keys, int rows, unsigned* counter);

__global__ void keys_decode_kernel(const long long* __restrict__ keys, int rows, const int* rows_dev,
                                   long long* idx_out, float* score_out);

__global__ void accept_offsets_kernel(const long long* __restrict__ draft, long long ld_draft,
                                      const long long* __restrict__ target, long long ld_target, int n_seq,
                                      int n_draft, int commit_extra, int* accept, int* offsets);

__global__ void pack_rows_kernel(const __nv_bfloat16* __restrict__ hidden, long long ld_seq, long long ld_row,
                                 int n_seq, int P, int H, const int* __restrict__ accept,
                                 const int* __restrict__ offsets, __nv_bfloat16* packed, long long ld_packed,
                                 int* row_pos);

__global__ void rnn_recurrence_kernel(const float* __restrict__ pre, int splits, long long split_stride,
                                      long long ld_pre, const __nv_bfloat16* __restrict__ w_s, const float* __restrict__ bias,
                                      const float* __restrict__ alpha, int n_seq, int T, int r,
                                      __nv_bfloat16* s_scaled, __nv_bfloat16* s_out, long long* keys,
                                      unsigned* counter);

__global__ void wait_selftest_kernel(int* status, unsigned long long limit_ns, unsigned long long* waited_ns);

inline size_t rnn_smem_bytes(int r) { return (size_t)(r / 2) * r * 4 + (size_t)kRnnSeqs * r * 4; }

}  // namespace dels
