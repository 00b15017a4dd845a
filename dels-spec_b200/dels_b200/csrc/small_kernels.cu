// Small SIMT kernels around the tensor-core scorer (sm_100a):
//   * rank-state finalisation after the split-K rank projection (a6),
//   * packed-key initialisation and decoding (a3 / cross-rank combine),
//   * ragged acceptance lengths + packed row offsets (a11) and the row gather that
//     packs accepted draft rows for the scorer,
//   * the input-projected RNN recurrence of the low-rank local head.
#include "small_kernels.cuh"

namespace dels {

// -----------------------------------------------------------------------------------
// Rank projection epilogue.  Reference: code/kernel/dels.py:437-439 —
//   rank_state = F.linear(h, W_rank)            (bf16 output, fp32 accumulation)
//   rank_state = F.silu(rank_state)             (optional, bf16 in/out)
// and the low-rank logit is scaled by alpha_p (code/kernel/dels.py:68).  Here the sum
// over split-K partials gives the fp32 accumulator; it is rounded to bf16 exactly like
// F.linear's output, optionally passed through SiLU and rounded again, and then
// alpha_p * s is rounded to bf16 so the scorer can add it to the long logits inside
// the same tensor-core accumulator.
// -----------------------------------------------------------------------------------
__global__ void rank_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                     long long ld_part, int rows, int r, int activation, const float* __restrict__ alpha,
                                     int n_pos, const int* __restrict__ row_pos, __nv_bfloat16* s_out,
                                     __nv_bfloat16* s_scaled, long long* keys, unsigned* counter) {
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  const long long total = (long long)rows * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / r);
    const long long pi = (long long)row * ld_part + (i - (long long)row * r);
    float acc = 0.0f;
    for (int s = 0; s < splits; ++s) acc += partials[s * split_stride + pi];
    float x = __bfloat162float(__float2bfloat16_rn(acc));
    if (activation == DELS_ACT_SILU) {
      x = __bfloat162float(__float2bfloat16_rn(x / (1.0f + expf(-x))));
    }
    if (s_out != nullptr) s_out[i] = __float2bfloat16_rn(x);
    const float a = alpha != nullptr ? alpha[row_position(row_pos, row, n_pos)] : 1.0f;
    s_scaled[i] = __float2bfloat16_rn(a * x);
    if (keys != nullptr && (i % r) == 0) keys[row] = kKeyEmpty;
  }
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
}

// -----------------------------------------------------------------------------------
// Domino correction-MLP hidden layer after the split-K projection s = W_s h:
// s_scaled = bf16(alpha[0] * SiLU(z + bf16(s))), SiLU in fp32 (code/kernel/domino.py:92-97,
// :113, :422), the same arithmetic as rank_gemv_kernel's addend path; keys reset.
// -----------------------------------------------------------------------------------
__global__ void correction_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                           long long ld_part, int rows, int m, const __nv_bfloat16* __restrict__ z,
                                           long long ld_z, const float* __restrict__ alpha, __nv_bfloat16* s_scaled,
                                           long long* keys, unsigned* counter) {
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  const long long total = (long long)rows * m;
  const float a = alpha != nullptr ? alpha[0] : 1.0f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / m);
    const int col = (int)(i - (long long)row * m);
    const long long pi = (long long)row * ld_part + col;
    float acc = 0.0f;
    for (int sp = 0; sp < splits; ++sp) acc += partials[sp * split_stride + pi];
    const float pre = __bfloat162float(z[(long long)row * ld_z + col]) + __bfloat162float(__float2bfloat16_rn(acc));
    s_scaled[i] = __float2bfloat16_rn(a * (pre / (1.0f + expf(-pre))));
    if (keys != nullptr && col == 0) keys[row] = kKeyEmpty;
  }
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
}

// -----------------------------------------------------------------------------------
// F.linear epilogue: out[row, n] = bf16(sum of the split-K partials + bias[n]).  The bias
// joins the fp32 accumulator before the single rounding, like the bias epilogue of the
// bf16 GEMM behind F.linear (code/kernel/domino.py:404-408, :325-327).
// -----------------------------------------------------------------------------------
__global__ void linear_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                       long long ld_part, int rows, int n, const __nv_bfloat16* __restrict__ bias,
                                       __nv_bfloat16* out, long long ld_out) {
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  const long long total = (long long)rows * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / n);
    const int col = (int)(i - (long long)row * n);
    const long long pi = (long long)row * ld_part + col;
    float acc = 0.0f;
    for (int s = 0; s < splits; ++s) acc += partials[s * split_stride + pi];
    if (bias != nullptr) acc += __bfloat162float(bias[col]);
    out[(long long)row * ld_out + col] = __float2bfloat16_rn(acc);
  }
}

__global__ void keys_init_kernel(long long* keys, int rows, unsigned* counter) {
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x)
    keys[i] = kKeyEmpty;
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
}

__global__ void keys_decode_kernel(const long long* __restrict__ keys, int rows, const int* rows_dev,
                                   long long* idx_out, float* score_out) {
  pdl_wait();
  int n = rows;
  if (rows_dev != nullptr) {
    const int d = *rows_dev;
    n = d < 0 ? 0 : (d < rows ? d : rows);
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const long long k = keys[i];
    if (idx_out != nullptr) idx_out[i] = (long long)key_index(k);
    if (score_out != nullptr) score_out[i] = key_score(k);
  }
}

// -----------------------------------------------------------------------------------
// Acceptance.  Reference: code/dflash.py:645-651 —
//   acceptance_length = (verify_ids[:, 1:] == posterior[:, :-1]).cumprod(dim=1).sum(dim=1)
// i.e. the length of the longest prefix on which draft token j equals the target
// token j.  One warp per sequence: a ballot of mismatches and a find-first-set give
// the prefix length; a block-wide exclusive scan turns lengths into packed row
// offsets (offsets[0] = 0, offsets[n_seq] = total rows).  Offsets count
// accept + commit_extra rows per sequence (commit_extra = 1 counts the bonus token
// that the decode loop commits, code/dflash.py:652-660).
// -----------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) accept_offsets_kernel(const long long* __restrict__ draft,
                                                              long long ld_draft,
                                                              const long long* __restrict__ target,
                                                              long long ld_target, int n_seq, int n_draft,
                                                              int commit_extra, int* accept, int* offsets) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  // Pass 1: accept lengths.
  for (int b = warp; b < n_seq; b += nwarps) {
    int len = 0;
    bool done = false;
    for (int j0 = 0; j0 < n_draft && !done; j0 += 32) {
      const int j = j0 + lane;
      bool mismatch = true;
      if (j < n_draft) mismatch = draft[(long long)b * ld_draft + j] != target[(long long)b * ld_target + j];
      const unsigned mm = __ballot_sync(0xFFFFFFFFu, mismatch);
      if (mm != 0u) {
        len = j0 + __ffs(mm) - 1;
        done = true;
      }
    }
    if (!done) len = n_draft;
    if (lane == 0) accept[b] = len;
  }
  __syncthreads();
  // Pass 2: exclusive scan of (accept + commit_extra) in chunks of blockDim.x.
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n_seq; base += blockDim.x) {
    const int b = base + threadIdx.x;
    const int v = (b < n_seq) ? accept[b] + commit_extra : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = (lane < nwarps) ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nwarps) warp_sums[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    const int warp_prefix = (warp > 0) ? warp_sums[warp - 1] : 0;
    const int excl = carry + warp_prefix + x - v;
    if (b < n_seq) offsets[b] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) offsets[n_seq] = carry;
}

// Gather the accepted rows of a [n_seq, P, H] hidden tensor into a packed
// [total, H] buffer (row offsets[b] + j holds hidden[b, j]) and record each packed
// row's draft position j (which selects alpha_j / beta_j).  One CTA per (b, j) slot.
__global__ void pack_rows_kernel(const __nv_bfloat16* __restrict__ hidden, long long ld_seq, long long ld_row,
                                 int n_seq, int P, int H, const int* __restrict__ accept,
                                 const int* __restrict__ offsets, __nv_bfloat16* packed, long long ld_packed,
                                 int* row_pos) {
  const int slot = blockIdx.x;
  const int b = slot / P, j = slot % P;
  if (b >= n_seq) return;
  if (j >= accept[b]) return;
  const long long dst_row = offsets[b] + j;
  const __nv_bfloat16* src = hidden + b * ld_seq + j * ld_row;
  __nv_bfloat16* dst = packed + dst_row * ld_packed;
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0 && (H % 8) == 0;
  if (vec) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
  }
  if (threadIdx.x == 0 && row_pos != nullptr) row_pos[dst_row] = j;
}

// -----------------------------------------------------------------------------------
// Input-projected RNN local head (no counterpart in the reference,
// which only has the GRU form of code/kernel/dels.py:359-373):
//   s_t = tanh(W_in x_t + W_s s_{t-1} + b),  s_0 = 0,  t = 0..T-1
// The input projection W_in x_t for all t comes in as split-K fp32 partials from the
// tensor-core GEMM (it does not depend on the recurrence).  The recurrence runs in
// fp32 with W_s (bf16) resident in shared memory, transposed and packed in pairs so
// that thread i reads W_s[i][j], W_s[i][j+1] with one conflict-free 32-bit load.
// Output: alpha_t * s_t rounded to bf16 (the scorer's segment-1 operand) and
// optionally s_t itself.  Each CTA runs kRnnSeqs sequences; thread i owns state i.
// -----------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rnn_recurrence_kernel(
    const float* __restrict__ pre, int splits, long long split_stride, long long ld_pre,
    const __nv_bfloat16* __restrict__ w_s,
    const float* __restrict__ bias, const float* __restrict__ alpha, int n_seq, int T, int r,
    __nv_bfloat16* s_scaled, __nv_bfloat16* s_out, long long* keys, unsigned* counter) {
  extern __shared__ uint8_t smem_raw[];
  // wt2[(j/2) * r + i] = (W_s[i][j], W_s[i][j+1]) as a bf16 pair.
  uint32_t* wt2 = reinterpret_cast<uint32_t*>(smem_raw);
  float* state = reinterpret_cast<float*>(smem_raw + (size_t)(r / 2) * r * 4);  // [kRnnSeqs][r]
  const int i = threadIdx.x;
  const int seq0 = blockIdx.x * kRnnSeqs;

  // Thread ii copies row ii of W_s: its (j, j+1) pairs are the row's 32-bit words, read 16
  // bytes at a time and written to wt2[jp][ii] (consecutive threads, consecutive banks).
  if ((r % 8) == 0 && (reinterpret_cast<uintptr_t>(w_s) & 15u) == 0) {
    for (int ii = threadIdx.x; ii < r; ii += blockDim.x) {
      const uint4* row = reinterpret_cast<const uint4*>(w_s + (long long)ii * r);
      for (int c = 0; c < r / 8; ++c) {
        const uint4 v = __ldg(row + c);
        wt2[(4 * c + 0) * r + ii] = v.x;
        wt2[(4 * c + 1) * r + ii] = v.y;
        wt2[(4 * c + 2) * r + ii] = v.z;
        wt2[(4 * c + 3) * r + ii] = v.w;
      }
    }
  } else {
    for (int e = threadIdx.x; e < (r / 2) * r; e += blockDim.x) {
      const int jp = e / r, ii = e % r;
      const uint16_t lo = reinterpret_cast<const uint16_t*>(w_s)[(long long)ii * r + 2 * jp];
      const uint16_t hi = reinterpret_cast<const uint16_t*>(w_s)[(long long)ii * r + 2 * jp + 1];
      wt2[e] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
  }
  for (int e = threadIdx.x; e < kRnnSeqs * r; e += blockDim.x) state[e] = 0.0f;
  if (keys != nullptr) {
    for (int e = threadIdx.x; e < kRnnSeqs * T; e += blockDim.x) {
      const int q = seq0 + e / T;
      if (q < n_seq) keys[(long long)q * T + e % T] = kKeyEmpty;
    }
  }
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
  __syncthreads();

  const float b_i = (bias != nullptr && i < r) ? bias[i] : 0.0f;
  for (int t = 0; t < T; ++t) {
    // This step's input projection: the first kPreAhead split-K partials of every
    // sequence are loaded as independent loads before the recurrent dot products and
    // summed after them (in split order), so one L2 round trip overlaps the dot products
    // instead of a chain of dependent ones per split.
    constexpr int kPreAhead = 4;
    const float a_t = alpha != nullptr ? alpha[t] : 1.0f;
    float pv[kRnnSeqs][kPreAhead];
#pragma unroll
    for (int q = 0; q < kRnnSeqs; ++q) {
      const int seq = seq0 + q;
      const bool ok = i < r && seq < n_seq;
      const long long off = ((long long)seq * T + t) * ld_pre + i;
#pragma unroll
      for (int j = 0; j < kPreAhead; ++j) pv[q][j] = (ok && j < splits) ? pre[j * split_stride + off] : 0.0f;
    }
    float g[kRnnSeqs];
#pragma unroll
    for (int q = 0; q < kRnnSeqs; ++q) g[q] = 0.0f;
    if (i < r) {
#pragma unroll 4
      for (int jp = 0; jp < r / 2; ++jp) {
        const uint32_t w = wt2[jp * r + i];
        const float w0 = bf16_lo(w), w1 = bf16_hi(w);
#pragma unroll
        for (int q = 0; q < kRnnSeqs; ++q) {
          const float2 sv = reinterpret_cast<const float2*>(state + q * r)[jp];
          g[q] = fmaf(w0, sv.x, g[q]);
          g[q] = fmaf(w1, sv.y, g[q]);
        }
      }
    }
    __syncthreads();  // everyone has read s_{t-1}
    if (i < r) {
#pragma unroll
      for (int q = 0; q < kRnnSeqs; ++q) {
        const int seq = seq0 + q;
        if (seq < n_seq) {
          const long long row = (long long)seq * T + t;
          float p = 0.0f;
#pragma unroll
          for (int j = 0; j < kPreAhead; ++j)
            if (j < splits) p += pv[q][j];
          for (int sp = kPreAhead; sp < splits; ++sp) p += pre[sp * split_stride + row * ld_pre + i];
          const float st = tanhf(p + g[q] + b_i);
          state[q * r + i] = st;
          s_scaled[row * r + i] = __float2bfloat16_rn(a_t * st);
          if (s_out != nullptr) s_out[row * r + i] = __float2bfloat16_rn(st);
        }
      }
    }
    __syncthreads();
  }
}

// -----------------------------------------------------------------------------------
// Self-test of the bounded wait that every tensor-core kernel uses.  Thread 0 waits on
// an mbarrier that nothing ever completes, with a short limit: the wait must give up,
// raise the CTA's abort flag and record DELS_ERR_DEVICE_TIMEOUT.  Thread 32 (another
// warp) waits on a second such barrier with the full limit and must leave as soon as
// it sees the abort flag — the path the producer / MMA / epilogue roles take when one
// of them times out.  Both report how long they waited.
// -----------------------------------------------------------------------------------
__global__ void wait_selftest_kernel(int* status, unsigned long long limit_ns, unsigned long long* waited_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 || threadIdx.x == 32) {
    const int which = threadIdx.x == 0 ? 0 : 1;
    const unsigned long long t0 = globaltimer_ns();
    const bool ok = mbar_wait(smem_u32(&bars[which]), 0u, &abort_flag, status,
                              which == 0 ? limit_ns : kWaitLimitNs);
    waited_ns[which] = ok ? 0ull : (globaltimer_ns() - t0);
  }
}

}  // namespace dels
