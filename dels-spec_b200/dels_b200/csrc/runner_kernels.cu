// Small-batch kernels of the greedy suffix rollout that DeLSGraphRunner /
// MarkovDeLSGraphRunner capture in a CUDA graph (B = 1 .. a few dozen rows):
//
//   * gru_step_kernel      — gi = table[token], gh = bf16(W_hh h + b_hh), then the GRU
//                            gates in fp32 and h' stored as bf16, in one launch
//                            (code/kernel/dels.py:359-373 + the Triton cell :140-211 +
//                            the table gather :432, :461);
//   * rank_gemv_kernel     — s = bf16(act(bf16(W_rank h + b))), s_scaled = bf16(alpha s),
//                            and the packed keys reset (code/kernel/dels.py:437-443); for the
//                            Domino correction MLP, s = SiLU(z + bf16(W_s h)) in fp32
//                            (code/kernel/domino.py:422, :92-97);
//   * gather_scaled_kernel — Markov rank state s = embedding[token], s_scaled = bf16(alpha s)
//                            (code/kernel/markov_dels.py:288).
//
// At these batch sizes every weight matrix is read once per step and each element is
// used B times, so the kernels are memory-bound GEMVs: warps stream weight rows with
// coalesced 16-byte loads (lane l owns elements 8l..8l+7 of every 256-element chunk),
// the B input rows sit in shared memory, and a butterfly shuffle finishes each dot
// product.
#include "runner_kernels.cuh"

namespace dels {

namespace {

// One weight row, lane l holding elements 8l..8l+7 of each 256-element chunk.  The
// first kRowPre chunks are loaded into registers ahead of time (before the input rows
// are staged), so a warp has its whole row in flight at once instead of one 16-byte
// load per lane per round trip.
constexpr int kRowPre = 4;

struct RowPrefetch {
  uint4 w[kRowPre];
};

__device__ __forceinline__ void row_prefetch(const __nv_bfloat16* __restrict__ wrow, int K, int lane,
                                             RowPrefetch& p) {
#pragma unroll
  for (int i = 0; i < kRowPre; ++i) {
    const int k = lane * 8 + i * 256;
    p.w[i] = k < K ? __ldg(reinterpret_cast<const uint4*>(wrow + k)) : make_uint4(0u, 0u, 0u, 0u);
  }
}

// acc[b] += w[k..k+7] . xs[b][k..k+7] for the nb staged rows
template <int MAXB>
__device__ __forceinline__ void dot_chunk(const uint4 w, const __nv_bfloat16* xs, int ldx, int nb, int k,
                                          float (&acc)[MAXB]) {
  const float w0 = bf16_lo(w.x), w1 = bf16_hi(w.x), w2 = bf16_lo(w.y), w3 = bf16_hi(w.y);
  const float w4 = bf16_lo(w.z), w5 = bf16_hi(w.z), w6 = bf16_lo(w.w), w7 = bf16_hi(w.w);
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    if (b < nb) {
      const uint4 x = *reinterpret_cast<const uint4*>(xs + b * ldx + k);
      float a = acc[b];
      a = fmaf(w0, bf16_lo(x.x), a);
      a = fmaf(w1, bf16_hi(x.x), a);
      a = fmaf(w2, bf16_lo(x.y), a);
      a = fmaf(w3, bf16_hi(x.y), a);
      a = fmaf(w4, bf16_lo(x.z), a);
      a = fmaf(w5, bf16_hi(x.z), a);
      a = fmaf(w6, bf16_lo(x.w), a);
      a = fmaf(w7, bf16_hi(x.w), a);
      acc[b] = a;
    }
  }
}

// dot products of one weight row (bf16, length K, first chunks already in `pre`) with
// `nb` bf16 rows staged in shared memory (row stride ldx elements); the full sums end
// up in every lane.  Chunks past the prefetched ones stream in batches of kRowPre.
template <int MAXB>
__device__ __forceinline__ void warp_row_dots(const RowPrefetch& pre, const __nv_bfloat16* __restrict__ wrow,
                                              const __nv_bfloat16* xs, int ldx, int nb, int K, int lane,
                                              float (&acc)[MAXB]) {
#pragma unroll
  for (int b = 0; b < MAXB; ++b) acc[b] = 0.0f;
#pragma unroll
  for (int i = 0; i < kRowPre; ++i) {
    const int k = lane * 8 + i * 256;
    if (k < K) dot_chunk<MAXB>(pre.w[i], xs, ldx, nb, k, acc);
  }
  for (int k0 = kRowPre * 256; k0 < K; k0 += kRowPre * 256) {
    RowPrefetch more;
    row_prefetch(wrow + k0, K - k0, lane, more);
#pragma unroll
    for (int i = 0; i < kRowPre; ++i) {
      const int k = k0 + lane * 8 + i * 256;
      if (k < K) dot_chunk<MAXB>(more.w[i], xs, ldx, nb, k, acc);
    }
  }
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    float a = acc[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    acc[b] = a;
  }
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }


}  // namespace

// One CTA per kGruCols hidden units, one warp per gate row of those units (the CTA has
// 3 * kGruCols warps); B rows in chunks of MAXB.  Each warp loads its W_hh row before h is
// staged, so the weight stream and the h gather overlap.
template <int MAXB>
__global__ void __launch_bounds__(kGruThreads, 2) gru_step_kernel(const long long* __restrict__ tokens,
                                                               long long tok_stride, int token_keys,
                                                               const __nv_bfloat16* __restrict__ table,
                                                               long long ld_table,
                                                               const __nv_bfloat16* __restrict__ w_hh,
                                                               const __nv_bfloat16* __restrict__ b_hh,
                                                               const __nv_bfloat16* h_in, __nv_bfloat16* h_out, int B,
                                                               int G, int V, int* status) {
  extern __shared__ uint4 smem4[];
  __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(smem4);  // [MAXB][G]
  float* gh_s = reinterpret_cast<float*>(hs + (size_t)MAXB * G);  // [3][kGruCols][MAXB]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g0 = blockIdx.x * kGruCols;
  // this warp's gate row: gate = warp / kGruCols, unit g0 + warp % kGruCols
  const int gate = warp / kGruCols, c_w = warp % kGruCols;
  const bool has_row = gate < 3 && g0 + c_w < G;
  const __nv_bfloat16* wrow = w_hh + (long long)(gate * G + g0 + c_w) * G;
  RowPrefetch pre;
  if (has_row) row_prefetch(wrow, G, lane, pre);  // weights only: safe before the wait
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  for (int b0 = 0; b0 < B; b0 += MAXB) {
    const int nb = min(MAXB, B - b0);
    __syncthreads();
    // stage h_in rows (zeros when h_in is NULL: the rollout's initial state)
    for (int e = threadIdx.x; e < nb * G / 8; e += blockDim.x) {
      const int b = e / (G / 8), k8 = e % (G / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (h_in != nullptr) v = *reinterpret_cast<const uint4*>(h_in + (long long)(b0 + b) * G + k8 * 8);
      reinterpret_cast<uint4*>(hs + (size_t)b * G)[k8] = v;
    }
    __syncthreads();
    // gh for the gate row {g, G + g, 2G + g} this warp owns
    if (has_row) {
      float acc[MAXB];
      warp_row_dots<MAXB>(pre, wrow, hs, G, nb, G, lane, acc);
      if (lane == 0) {
        const int g = g0 + c_w;
        const float bias = b_hh != nullptr ? __bfloat162float(b_hh[gate * G + g]) : 0.0f;
#pragma unroll
        for (int b = 0; b < MAXB; ++b)
          if (b < nb) gh_s[(gate * kGruCols + c_w) * MAXB + b] = bf16r(acc[b] + bias);
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nb * kGruCols; e += blockDim.x) {
      const int b = e / kGruCols, c = e % kGruCols;
      const int g = g0 + c;
      if (g >= G) continue;
      long long tok = tokens[(long long)(b0 + b) * tok_stride];
      if (token_keys) tok = (long long)key_index(tok);  // the scorer's packed (score, index) key
      if (tok < 0 || tok >= V) {
        if (status != nullptr) atomicCAS(status, 0, DELS_ERR_INVALID_ARG);
        tok = tok < 0 ? 0 : V - 1;
      }
      const __nv_bfloat16* gi = table + tok * ld_table;
      const float gi_r = __bfloat162float(gi[g]);
      const float gi_z = __bfloat162float(gi[G + g]);
      const float gi_n = __bfloat162float(gi[2 * G + g]);
      const float gh_r = gh_s[(0 * kGruCols + c) * MAXB + b];
      const float gh_z = gh_s[(1 * kGruCols + c) * MAXB + b];
      const float gh_n = gh_s[(2 * kGruCols + c) * MAXB + b];
      const float h = __bfloat162float(hs[(size_t)b * G + g]);
      h_out[(long long)(b0 + b) * G + g] = __float2bfloat16_rn(gru_unit(gi_r, gi_z, gi_n, gh_r, gh_z, gh_n, h));
    }
  }
}

// One warp per output feature j (grid-stride), all B rows at once.  The warp's first
// weight row is loaded before x is staged.  With `addend` (the Domino correction MLP)
// the output is SiLU(addend + bf16(W x)) in fp32 instead of the rank activation.
template <int MAXB>
__global__ void __launch_bounds__(kGemvThreads) rank_gemv_kernel(
    const __nv_bfloat16* __restrict__ x, long long ld_x, const __nv_bfloat16* __restrict__ w, long long ld_w,
    const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ addend, long long ld_add, int B,
    int K, int r, int activation, const float* __restrict__ alpha, int n_pos, const int* __restrict__ row_pos,
    __nv_bfloat16* s_out, __nv_bfloat16* s_scaled, long long* keys, unsigned* counter, const GruGateSrc gate) {
  extern __shared__ uint4 smem4[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem4);  // [MAXB][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gwarp = blockIdx.x * (blockDim.x >> 5) + warp;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  RowPrefetch first;
  if (gwarp < r) row_prefetch(w + (long long)gwarp * ld_w, K, lane, first);  // weights only
  pdl_wait();
  // The next kernel (the rollout step's scorer) may launch now: its weight prefetch runs
  // before its own wait, so the Vr stream overlaps the gates and the projection below
  // (batch-1 runner call -6 %).  It reads what this kernel writes only after that wait.
  pdl_trigger();
  for (int b0 = 0; b0 < B; b0 += MAXB) {
    const int nb = min(MAXB, B - b0);
    __syncthreads();
    if (gate.table != nullptr) {
      // x = the GRU's new hidden state (K = G units), eight units per thread: every CTA
      // evaluates all of them from L2-resident inputs instead of waiting for a GRU kernel
      for (int e = threadIdx.x; e < nb * K / 8; e += blockDim.x) {
        const int b = e / (K / 8), k8 = e % (K / 8);
        const int row = b0 + b;
        const int G8 = K / 8;  // uint4 per gate block
        // gh and h do not depend on the token: their loads go out together with the token's
        // (one L2 round trip), ahead of the table row that the token selects
        const uint4* gh = reinterpret_cast<const uint4*>(gate.gh + (long long)row * gate.ld_gh) + k8;
        const uint4 hr = gh[0], hz = gh[G8], hn = gh[2 * G8];
        const uint4 hp = gate.h_in != nullptr
                             ? *(reinterpret_cast<const uint4*>(gate.h_in + (long long)row * K) + k8)
                             : make_uint4(0u, 0u, 0u, 0u);
        long long tok = gate.tokens[(long long)row * gate.tok_stride];
        if (gate.token_keys) tok = (long long)key_index(tok);  // the scorer's packed (score, index) key
        if (tok < 0 || tok >= gate.V) {
          if (gate.status != nullptr) atomicCAS(gate.status, 0, DELS_ERR_INVALID_ARG);
          tok = tok < 0 ? 0 : gate.V - 1;
        }
        const uint4* gi = reinterpret_cast<const uint4*>(gate.table + tok * gate.ld_table) + k8;
        const uint4 ir = __ldg(gi), iz = __ldg(gi + G8), in = __ldg(gi + 2 * G8);
        const uint32_t* a_r = &ir.x; const uint32_t* a_z = &iz.x; const uint32_t* a_n = &in.x;
        const uint32_t* b_r = &hr.x; const uint32_t* b_z = &hz.x; const uint32_t* b_n = &hn.x;
        const uint32_t* c_h = &hp.x;
        uint4 o;
        uint32_t* op = &o.x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = gru_unit(bf16_lo(a_r[q]), bf16_lo(a_z[q]), bf16_lo(a_n[q]), bf16_lo(b_r[q]),
                                    bf16_lo(b_z[q]), bf16_lo(b_n[q]), bf16_lo(c_h[q]));
          const float hi = gru_unit(bf16_hi(a_r[q]), bf16_hi(a_z[q]), bf16_hi(a_n[q]), bf16_hi(b_r[q]),
                                    bf16_hi(b_z[q]), bf16_hi(b_n[q]), bf16_hi(c_h[q]));
          op[q] = pack_bf16x2(lo, hi);
        }
        reinterpret_cast<uint4*>(xs + (size_t)b * K)[k8] = o;
        if (blockIdx.x == 0) reinterpret_cast<uint4*>(gate.h_out + (long long)row * K)[k8] = o;
      }
    } else {
      for (int e = threadIdx.x; e < nb * K / 8; e += blockDim.x) {
        const int b = e / (K / 8), k8 = e % (K / 8);
        reinterpret_cast<uint4*>(xs + (size_t)b * K)[k8] =
            *reinterpret_cast<const uint4*>(x + (long long)(b0 + b) * ld_x + k8 * 8);
      }
    }
    __syncthreads();
    for (int j = gwarp; j < r; j += nwarps) {
      const __nv_bfloat16* wrow = w + (long long)j * ld_w;
      RowPrefetch pre;
      if (j == gwarp) {
        pre = first;
      } else {
        row_prefetch(wrow, K, lane, pre);
      }
      float acc[MAXB];
      warp_row_dots<MAXB>(pre, wrow, xs, K, nb, K, lane, acc);
      if (lane < nb) {
        float a = 0.0f;
#pragma unroll
        for (int b = 0; b < MAXB; ++b)
          if (b == lane) a = acc[b];
        const int row = b0 + lane;
        const float bj = bias != nullptr ? __bfloat162float(bias[j]) : 0.0f;
        float s = bf16r(a + bj);
        if (addend != nullptr) {
          // correction MLP: SiLU(z + s) in fp32, not re-rounded (code/kernel/domino.py:92-97)
          const float pre = __bfloat162float(addend[(long long)row * ld_add + j]) + s;
          s = pre / (1.0f + expf(-pre));
        } else if (activation == DELS_ACT_SILU) {
          s = bf16r(s / (1.0f + expf(-s)));
        }
        if (s_out != nullptr) s_out[(long long)row * r + j] = __float2bfloat16_rn(s);
        const float al = alpha != nullptr ? alpha[row_position(row_pos, row, n_pos)] : 1.0f;
        s_scaled[(long long)row * r + j] = __float2bfloat16_rn(al * s);
      }
    }
  }
  if (keys != nullptr && blockIdx.x == 0) {
    for (int i = threadIdx.x; i < B; i += blockDim.x) keys[i] = kKeyEmpty;
  }
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
}

// Rows per shared-memory pass: the compile-time row count of the dot-product loops.  Rows
// past the batch are skipped under a predicate, and predicated-off FMAs still take issue
// slots, so a batch-1 rollout compiled for 16 rows would issue 16x the arithmetic it needs.
GruStepKernel gru_step_kernel_for(int rows_per_pass) {
  switch (rows_per_pass) {
    case 1: return gru_step_kernel<1>;
    case 2: return gru_step_kernel<2>;
    case 4: return gru_step_kernel<4>;
    case 8: return gru_step_kernel<8>;
    default: return gru_step_kernel<kRunnerMaxB>;
  }
}

RankGemvKernel rank_gemv_kernel_for(int rows_per_pass) {
  switch (rows_per_pass) {
    case 1: return rank_gemv_kernel<1>;
    case 2: return rank_gemv_kernel<2>;
    case 4: return rank_gemv_kernel<4>;
    case 8: return rank_gemv_kernel<8>;
    default: return rank_gemv_kernel<kRunnerMaxB>;
  }
}

// The GRU gates for batches where gh = bf16(W_hh h + b_hh) came from the tensor-core
// projection (dels_linear_bf16): one thread per (row, unit), the same gate arithmetic as
// gru_step_kernel.
__global__ void gru_gates_kernel(const long long* __restrict__ tokens, long long tok_stride, int token_keys,
                                 const __nv_bfloat16* __restrict__ table, long long ld_table,
                                 const __nv_bfloat16* __restrict__ gh, long long ld_gh, const __nv_bfloat16* h_in,
                                 __nv_bfloat16* h_out, int B, int G, int V, int* status) {
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < (long long)B * G;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / G), g = (int)(e % G);
    long long tok = tokens[(long long)b * tok_stride];
    if (token_keys) tok = (long long)key_index(tok);  // the scorer's packed (score, index) key
    if (tok < 0 || tok >= V) {
      if (status != nullptr) atomicCAS(status, 0, DELS_ERR_INVALID_ARG);
      tok = tok < 0 ? 0 : V - 1;
    }
    const __nv_bfloat16* gi = table + tok * ld_table;
    const __nv_bfloat16* ghb = gh + (long long)b * ld_gh;
    const float h = h_in != nullptr ? __bfloat162float(h_in[(long long)b * G + g]) : 0.0f;
    h_out[(long long)b * G + g] = __float2bfloat16_rn(
        gru_unit(__bfloat162float(gi[g]), __bfloat162float(gi[G + g]), __bfloat162float(gi[2 * G + g]),
                 __bfloat162float(ghb[g]), __bfloat162float(ghb[G + g]), __bfloat162float(ghb[2 * G + g]), h));
  }
}

// The GRU step after a tensor-core split-K projection of W_hh h_in: per (row, unit) the
// three gate columns' partial sums are added in split order, the bias joins the fp32 sum
// and the result is rounded to bf16 once (as dels_linear_bf16's finalisation writes gh),
// then the gates as gru_gates_kernel evaluates them.  The partials of a split group are
// loaded together, ahead of the sums.
__global__ void gru_finalize_kernel(const float* __restrict__ partials, int splits, long long split_stride,
                                    long long ld_part, const long long* __restrict__ tokens, long long tok_stride,
                                    int token_keys, const __nv_bfloat16* __restrict__ table, long long ld_table,
                                    const __nv_bfloat16* __restrict__ b_hh, const __nv_bfloat16* h_in,
                                    __nv_bfloat16* h_out, int B, int G, int V, int* status) {
  constexpr int kAhead = 4;
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < (long long)B * G;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / G), g = (int)(e % G);
    long long tok = tokens[(long long)b * tok_stride];
    if (token_keys) tok = (long long)key_index(tok);  // the scorer's packed (score, index) key
    const float h = h_in != nullptr ? __bfloat162float(h_in[(long long)b * G + g]) : 0.0f;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    for (int s0 = 0; s0 < splits; s0 += kAhead) {
      float v[3][kAhead];
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int q = 0; q < kAhead; ++q)
          v[j][q] = s0 + q < splits ? partials[(s0 + q) * split_stride + (long long)b * ld_part + j * G + g] : 0.0f;
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int q = 0; q < kAhead; ++q)
          if (s0 + q < splits) acc[j] += v[j][q];
    }
    float gh[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float a = acc[j];
      if (b_hh != nullptr) a += __bfloat162float(b_hh[j * G + g]);
      gh[j] = __bfloat162float(__float2bfloat16_rn(a));
    }
    if (tok < 0 || tok >= V) {
      if (status != nullptr) atomicCAS(status, 0, DELS_ERR_INVALID_ARG);
      tok = tok < 0 ? 0 : V - 1;
    }
    const __nv_bfloat16* gi = table + tok * ld_table;
    h_out[(long long)b * G + g] = __float2bfloat16_rn(gru_unit(__bfloat162float(gi[g]), __bfloat162float(gi[G + g]),
                                                               __bfloat162float(gi[2 * G + g]), gh[0], gh[1], gh[2], h));
  }
}

__global__ void gather_scaled_kernel(const long long* __restrict__ tokens, long long tok_stride, int token_keys,
                                     const __nv_bfloat16* __restrict__ emb, long long ld_emb,
                                     const float* __restrict__ alpha, int n_pos, int B, int r, int V,
                                     __nv_bfloat16* s_scaled, long long* keys, unsigned* counter, int* status) {
  pdl_wait();
  pdl_trigger();  // the next kernel reads our output only after its own wait
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < B * r; e += gridDim.x * blockDim.x) {
    const int b = e / r, j = e % r;
    long long tok = tokens[(long long)b * tok_stride];
    if (token_keys) tok = (long long)key_index(tok);  // the scorer's packed (score, index) key
    if (tok < 0 || tok >= V) {
      if (status != nullptr) atomicCAS(status, 0, DELS_ERR_INVALID_ARG);
      tok = tok < 0 ? 0 : V - 1;
    }
    const float a = alpha != nullptr ? alpha[b % n_pos] : 1.0f;
    s_scaled[e] = __float2bfloat16_rn(a * __bfloat162float(emb[tok * ld_emb + j]));
    if (keys != nullptr && j == 0) keys[b] = kKeyEmpty;
  }
  if (counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;
}

}  // namespace dels
