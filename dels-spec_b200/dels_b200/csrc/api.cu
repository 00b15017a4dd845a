// C ABI of the DeLS draft-scoring hot path: argument validation, tensor-map encoding,
// grid sizing and kernel launches.  Declarations and the contract of every entry
// point are in include/dels_b200.h.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <string>

#include "f32_score.cuh"
#include "runner_kernels.cuh"
#include "small_kernels.cuh"
#include "tc_gemm.cuh"
#include "tc_scorer_pair.cuh"
#include "tc_skinny.cuh"

using namespace dels;

namespace {

constexpr int kVersion = 1;
constexpr int kMaxDevices = 64;
// Split-K sizing of the projection GEMMs aims at this many CTAs (one B200 wave).
constexpr int kTargetCtas = 148;
// Scorer schedule: 16 row tiles (2048 rows, a 17.8 MB A panel at H + r = 4352) sweep
// the vocabulary together; the last partial wave's tiles are split 4 ways along N.
constexpr int kScorerGroupM = 16;
constexpr int kScorerTailSplit = 4;
// Paired scorer enabled (DELS_SCORER_PAIRS=0 in the environment selects the
// single-CTA scorer for every shape, e.g. to compare the two).
bool g_use_pairs = true;
// Skinny (rows as the MMA's N side) scorer for calls of at most kSkinnyMaxRows rows
// (DELS_SCORER_SKINNY=0 in the environment selects the 128-row tile kernel instead).
bool g_use_skinny = true;
constexpr int kSkinnyMaxRows = 32;
// K blocks per pipeline stage of the paired scorer (DELS_PAIR_KGROUP=1 or 2)
int g_pair_kgroup = 2;
constexpr int kSkinnyStageRows = 4;
// Programmatic dependent launch for the kernels of a rollout step (DELS_PDL=0 in the
// environment turns it off).
bool g_use_pdl = true;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DELS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define DELS_CHECK_LAUNCH(what)                    \
  do {                                             \
    cudaError_t e_ = cudaGetLastError();           \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Launch with programmatic stream serialisation: the kernel may start while the previous
// kernel in the stream finishes.  Only kernels that call pdl_wait() before touching the
// data of earlier kernels are launched this way.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_use_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define DELS_CHECK_PDL(what, ...)                    \
  do {                                               \
    cudaError_t e_ = (__VA_ARGS__);                  \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }

// ------------------------------------------------------------------ driver entry point
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

int ensure_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr)
    return fail(DELS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(g_encode_err));
  return DELS_OK;
}

// 2-D bf16 tensor map over a row-major [outer, inner] matrix with leading dimension
// `ld` elements, box = [box_outer rows, 64 elements], 128-byte swizzle, zero fill
// outside the extents (so K, row and vocab tails need no special casing).
int make_map_bf16(CUtensorMap* m, const void* ptr, long long inner, long long outer, long long ld, int box_outer) {
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DELS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for [%lld x %lld], ld %lld", (int)r, outer,
                inner, ld);
  return DELS_OK;
}

// 2-D fp32 tensor map, box = [box_outer rows, box_inner elements] (32 = 128 bytes), optional
// 128-byte swizzle, zero fill outside the extents.
int make_map_f32(CUtensorMap* m, const void* ptr, long long inner, long long outer, long long ld, int box_outer,
                 bool swizzle, int box_inner = 32) {
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DELS_ERR_CUDA, "cuTensorMapEncodeTiled (fp32) failed (%d) for [%lld x %lld], ld %lld", (int)r, outer,
                inner, ld);
  return DELS_OK;
}

// Epilogue-operand maps of the skinny scorer, no swizzle, zero fill outside the extents:
// base logits [rows, n] bf16 (row stride ld) in boxes of box_n x box_rows, and an fp32
// vector [n] (one row) in boxes of box_n.
int make_map_base_bf16(CUtensorMap* m, const void* ptr, long long n, long long rows, long long ld, int box_n,
                       int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_n, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DELS_ERR_CUDA, "cuTensorMapEncodeTiled (base) failed (%d) for [%lld x %lld], ld %lld", (int)r, rows, n,
                ld);
  return DELS_OK;
}

int make_map_vec_f32(CUtensorMap* m, const float* ptr, long long n, int box_n) {
  // one row of n; the row stride is never stepped but must be a multiple of 16 bytes
  cuuint64_t dims[2] = {(cuuint64_t)n, 1};
  cuuint64_t strides[1] = {(cuuint64_t)((n * 4 + 15) / 16 * 16)};
  cuuint32_t box[2] = {(cuuint32_t)box_n, 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DELS_ERR_CUDA, "cuTensorMapEncodeTiled (vector) failed (%d) for [%lld]", (int)r, n);
  return DELS_OK;
}

// ------------------------------------------------------------------ per-device state
struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int max_pairs = 0;  // co-resident 2-CTA clusters of the paired scorer
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

template <typename K>
cudaError_t set_smem(K kernel, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes attr;
  return cudaFuncGetAttributes(&attr, kernel);  // forces the module to load now
}

constexpr int kMaxSmem = 232448;

int init_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return fail(DELS_ERR_INVALID_ARG, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (g_dev[dev].ready) return DELS_OK;
  if (const char* env = getenv("DELS_SCORER_PAIRS")) g_use_pairs = env[0] != '0';
  if (const char* env = getenv("DELS_SCORER_SKINNY")) g_use_skinny = env[0] != '0';
  if (const char* env = getenv("DELS_PDL")) g_use_pdl = env[0] != '0';
  if (const char* env = getenv("DELS_PAIR_KGROUP")) g_pair_kgroup = env[0] == '1' ? 1 : 2;
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (prev != dev && (e = cudaSetDevice(dev)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int major = 0, minor = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int rc = DELS_OK;
  if (major != 10 || minor != 0) {
    rc = fail(DELS_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major, minor);
  } else {
#define SET(k, b)                                            \
  if (rc == DELS_OK && (e = set_smem(k, b)) != cudaSuccess) rc = cuda_fail(e, "kernel setup: " #k);
    SET((tc_gemm_kernel<256, kArgmax, false>), TcConfig<256>::kSmemBytes);
    SET((tc_gemm_kernel<256, kArgmax, true>), (TcConfig<256, true>::kSmemBytes));
    SET((tc_gemm_kernel<256, kStore, false>), TcConfig<256>::kSmemBytes);
    SET((tc_gemm_kernel<128, kStore, false>), TcConfig<128>::kSmemBytes);
    SET((tc_gemm_kernel<64, kStore, false>), TcConfig<64>::kSmemBytes);
    SET((tc_gemm_kernel<32, kStore, false>), TcConfig<32>::kSmemBytes);
    if (rc == DELS_OK && (e = f32_score_setup(kMaxSmem)) != cudaSuccess) rc = cuda_fail(e, "kernel setup: f32_score");
    SET((tc_scorer_pair_kernel<false, false, 1>), PairConfig::kSmemBytes);
    SET((tc_scorer_pair_kernel<true, false, 1>), PairConfig::kSmemBytes);
    SET((tc_scorer_pair_kernel<false, true, 1>), PairConfig::kSmemBytes);
    SET((tc_scorer_pair_kernel<false, false, 2>), PairConfig::kSmemBytes);
    SET((tc_scorer_pair_kernel<true, false, 2>), PairConfig::kSmemBytes);
    SET((tc_scorer_pair_kernel<false, true, 2>), PairConfig::kSmemBytes);
    SET((tc_skinny_kernel<16, 1>), (SkinnyConfig<16, false>::kSmemBytes));
    SET((tc_skinny_kernel<16, 4>), (SkinnyConfig<16, false>::kSmemBytes));
    SET((tc_skinny_kernel<16>), (SkinnyConfig<16, false>::kSmemBytes));
    SET((tc_skinny_gh_kernel<16, 1>), (SkinnyConfig<16, false>::kSmemBytes));
    SET((tc_skinny_gh_kernel<16, kSkinnyGhMaxB>), (SkinnyConfig<16, false>::kSmemBytes));
    SET((tc_skinny_gh_kernel<16, kSkinnyGhRows>), (SkinnyConfig<16, false>::kSmemBytes));
    SET((tc_skinny_staged_kernel<16>), SkinnyConfig<16>::kSmemBytes);
    SET((tc_skinny_kernel<32>), (SkinnyConfig<32, false>::kSmemBytes));
    SET((tc_skinny_staged_kernel<32>), SkinnyConfig<32>::kSmemBytes);
    SET(rnn_recurrence_kernel, kMaxSmem);
    SET(rank_finalize_kernel, 0);
    SET(keys_init_kernel, 0);
    SET(keys_decode_kernel, 0);
    SET(accept_offsets_kernel, 0);
    SET(pack_rows_kernel, 0);
    SET(f32_rank_kernel, 0);
    SET(f32_transpose_pass_kernel, 0);
    for (int rows_per_pass = 1; rows_per_pass <= kRunnerMaxB; rows_per_pass *= 2) {
      SET(gru_step_kernel_for(rows_per_pass), kMaxSmem);
      SET(rank_gemv_kernel_for(rows_per_pass), kMaxSmem);
    }
    SET(linear_finalize_kernel, 0);
    SET(correction_finalize_kernel, 0);
    SET(gather_scaled_kernel, 0);
    SET(gru_gates_kernel, 0);
    SET(gru_finalize_kernel, 0);
    SET(wait_selftest_kernel, 0);
#undef SET
  }
  if (rc == DELS_OK) {
    // A persistent grid of CTA pairs must fit on the device at once: ask the occupancy
    // calculator how many 2-CTA clusters can be resident (SMs pair up within a GPC).
    int pairs = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = PairConfig::kSmemBytes;
    e = cudaOccupancyMaxActiveClusters(&pairs, (const void*)tc_scorer_pair_kernel<false, false, 1>, &cfg);
    if (e != cudaSuccess || pairs <= 0) {
      cudaGetLastError();
      pairs = 0;  // the paired scorer is not used on this device
    }
    g_dev[dev].max_pairs = pairs < sms / 2 ? pairs : sms / 2;
    g_dev[dev].sm_count = sms;
    g_dev[dev].ready = true;
  }
  if (prev != dev) cudaSetDevice(prev);
  return rc;
}

// Current device, initialised on first use.
int current_device_state(DeviceState** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(DELS_ERR_INVALID_ARG, "device %d out of range", dev);
  if (!g_dev[dev].ready) {
    int rc = init_device(dev);
    if (rc != DELS_OK) return rc;
  }
  *out = &g_dev[dev];
  return DELS_OK;
}

struct WsHeader {
  unsigned* counter;
  int* status;
};

int ws_header(void* ws, size_t ws_bytes, size_t need, WsHeader* h) {
  if (ws == nullptr || ws_bytes < need)
    return fail(DELS_ERR_WORKSPACE, "workspace too small: %zu bytes given, %zu needed", ws ? ws_bytes : (size_t)0, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(DELS_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  h->counter = reinterpret_cast<unsigned*>(ws);
  h->status = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + 4);
  return DELS_OK;
}

int check_bf16_matrix(const char* name, const void* p, long long ld, long long k) {
  if (p == nullptr) return fail(DELS_ERR_INVALID_ARG, "%s is NULL", name);
  if (!aligned16(p)) return fail(DELS_ERR_ALIGNMENT, "%s must be 16-byte aligned", name);
  if (ld < k || (ld % 8) != 0)
    return fail(DELS_ERR_ALIGNMENT, "%s: leading dimension %lld must be >= %lld and a multiple of 8", name, ld, k);
  return DELS_OK;
}

// ------------------------------------------------------------------ tensor-core launches
struct TcOperands {
  const void* a0 = nullptr;
  long long lda0 = 0;
  const void* b0 = nullptr;
  long long ldb0 = 0;
  int K0 = 0;
  const void* a1 = nullptr;
  long long lda1 = 0;
  const void* b1 = nullptr;
  long long ldb1 = 0;
  int K1 = 0;
  int m_extent = 0;  // rows of A (capacity)
  int n_extent = 0;  // rows of B
};

template <int BN, int MODE, bool VB>
int launch_tc(const TcOperands& op, TcArgs args, int sm_count, cudaStream_t st) {
  int rc = ensure_encode();
  if (rc != DELS_OK) return rc;
  // B maps come in two box heights: BN rows for whole tiles and BN / tail_split rows
  // for the split tiles of the last partial wave.
  const int tail_rows = BN / (args.tail_split > 1 ? args.tail_split : 1);
  CUtensorMap ma0, mb0, ma1, mb1, mb0t, mb1t;
  if (op.K1 > 0) {
    if ((rc = make_map_bf16(&ma1, op.a1, op.K1, op.m_extent, op.lda1, kBM)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb1, op.b1, op.K1, op.n_extent, op.ldb1, BN)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb1t, op.b1, op.K1, op.n_extent, op.ldb1, tail_rows)) != DELS_OK) return rc;
  }
  if (op.K0 > 0) {
    if ((rc = make_map_bf16(&ma0, op.a0, op.K0, op.m_extent, op.lda0, kBM)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb0, op.b0, op.K0, op.n_extent, op.ldb0, BN)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb0t, op.b0, op.K0, op.n_extent, op.ldb0, tail_rows)) != DELS_OK) return rc;
  } else {
    ma0 = ma1;
    mb0 = mb1;
    mb0t = mb1t;
  }
  if (op.K1 == 0) {
    ma1 = ma0;
    mb1 = mb0;
    mb1t = mb0t;
  }
  args.kb0 = cdiv(op.K0, kBK);
  args.kb1 = cdiv(op.K1, kBK);
  const long long tiles = (long long)cdiv(op.m_extent, kBM) * cdiv(op.n_extent, BN) * args.k_splits;
  // With fewer tiles than SMs, split tiles (tail_split ways) so more SMs take part.
  const long long want = tiles < sm_count ? tiles * (args.tail_split > 1 ? args.tail_split : 1) : tiles;
  const int grid = (int)(want < sm_count ? want : sm_count);
  if (grid <= 0) return DELS_OK;
  constexpr int smem = TcConfig<BN, VB && MODE == kArgmax>::kSmemBytes;
  DELS_CHECK_PDL("tc_gemm_kernel launch", launch_pdl(tc_gemm_kernel<BN, MODE, VB>, dim3(grid),
      dim3(kTcThreads), smem, st, ma0, mb0, ma1, mb1, mb0t, mb1t, args));
  return DELS_OK;
}

// The skinny scorer: weight maps (W, Vr) in 64 x 128 boxes as the MMA's A operand, row
// maps (h, s) in 64 x NB boxes as its B operand; one persistent CTA per SM.
template <int NB, bool SB, bool GH = false>
int launch_skinny(const TcOperands& op, TcArgs args, int sm_count, cudaStream_t st) {
  int rc = ensure_encode();
  if (rc != DELS_OK) return rc;
  CUtensorMap wa0, rb0, wa1, rb1;
  if (op.K1 > 0) {
    if ((rc = make_map_bf16(&wa1, op.b1, op.K1, op.n_extent, op.ldb1, kSkinnyBM)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&rb1, op.a1, op.K1, op.m_extent, op.lda1, NB)) != DELS_OK) return rc;
  }
  if (op.K0 > 0) {
    if ((rc = make_map_bf16(&wa0, op.b0, op.K0, op.n_extent, op.ldb0, kSkinnyBM)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&rb0, op.a0, op.K0, op.m_extent, op.lda0, NB)) != DELS_OK) return rc;
  } else {
    wa0 = wa1;
    rb0 = rb1;
  }
  if (op.K1 == 0) {
    wa1 = wa0;
    rb1 = rb0;
  }
  args.kb0 = cdiv(op.K0, kBK);
  args.kb1 = cdiv(op.K1, kBK);
  // the epilogue operands (base logits when TMA can address them, prior): fetched by the
  // producer; unused maps are copies of a weight map
  CUtensorMap mbase = wa1, mprior = wa1;
  if (SB && args.base != nullptr &&
      (rc = make_map_base_bf16(&mbase, args.base, op.n_extent, op.m_extent, args.ld_base, kSkinnyBM, NB)) != DELS_OK)
    return rc;
  if (SB && args.prior != nullptr && (rc = make_map_vec_f32(&mprior, args.prior, op.n_extent, kSkinnyBM)) != DELS_OK)
    return rc;
  const int tiles = cdiv(op.n_extent, kSkinnyBM);
  const int grid = tiles < sm_count ? tiles : sm_count;
  if (grid <= 0) return DELS_OK;
  if constexpr (GH) {
    // the epilogue and the helper GEMV compiled for the fewest rows that hold the batch
    auto kernel = args.m_rows <= 1 ? tc_skinny_gh_kernel<NB, 1>
                  : (args.m_rows <= kSkinnyGhMaxB ? tc_skinny_gh_kernel<NB, kSkinnyGhMaxB>
                                                  : tc_skinny_gh_kernel<NB, kSkinnyGhRows>);
    DELS_CHECK_PDL("tc_skinny_gh_kernel launch", launch_pdl(kernel, dim3(grid), dim3(kSkinnyGhThreads),
        SkinnyConfig<NB, false>::kSmemBytes, st, wa0, rb0, wa1, rb1, args));
  } else if constexpr (SB) {
    DELS_CHECK_PDL("tc_skinny_staged_kernel launch", launch_pdl(tc_skinny_staged_kernel<NB>, dim3(grid),
        dim3(kTcThreads), SkinnyConfig<NB>::kSmemBytes, st, wa0, rb0, wa1, rb1, mbase, mprior, args));
  } else {
    // the 16-column kernel's epilogue compiled for the fewest rows that hold the batch (1, 4, 16)
    auto kernel = tc_skinny_kernel<NB, NB>;
    if constexpr (NB == 16) {
      if (args.m_rows <= 1) kernel = tc_skinny_kernel<NB, 1>;
      else if (args.m_rows <= 4) kernel = tc_skinny_kernel<NB, 4>;
    }
    DELS_CHECK_PDL("tc_skinny_kernel launch", launch_pdl(kernel, dim3(grid), dim3(kTcThreads),
        SkinnyConfig<NB, false>::kSmemBytes, st, wa0, rb0, wa1, rb1, args));
  }
  return DELS_OK;
}

// The paired (cta_group::2) scorer: 256-row pair tiles, each CTA stages 128 rows of A
// and half of the 256-token B tile (128 rows; 32 rows for the split tail units).
template <bool VB, bool STORE = false>
int launch_scorer_pair(const TcOperands& op, TcArgs args, int max_pairs, cudaStream_t st) {
  int rc = ensure_encode();
  if (rc != DELS_OK) return rc;
  constexpr int half = PairConfig::kHalfBN;
  const int tail_half = PairConfig::BN / (args.tail_split > 1 ? args.tail_split : 1) / 2;
  CUtensorMap ma0, mb0, ma1, mb1, mb0t, mb1t;
  if (op.K1 > 0) {
    if ((rc = make_map_bf16(&ma1, op.a1, op.K1, op.m_extent, op.lda1, kBM)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb1, op.b1, op.K1, op.n_extent, op.ldb1, half)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb1t, op.b1, op.K1, op.n_extent, op.ldb1, tail_half)) != DELS_OK) return rc;
  }
  if (op.K0 > 0) {
    if ((rc = make_map_bf16(&ma0, op.a0, op.K0, op.m_extent, op.lda0, kBM)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb0, op.b0, op.K0, op.n_extent, op.ldb0, half)) != DELS_OK) return rc;
    if ((rc = make_map_bf16(&mb0t, op.b0, op.K0, op.n_extent, op.ldb0, tail_half)) != DELS_OK) return rc;
  } else {
    ma0 = ma1;
    mb0 = mb1;
    mb0t = mb1t;
  }
  if (op.K1 == 0) {
    ma1 = ma0;
    mb1 = mb0;
    mb1t = mb0t;
  }
  args.kb0 = cdiv(op.K0, kBK);
  args.kb1 = cdiv(op.K1, kBK);
  const long long tiles = (long long)cdiv(op.m_extent, 2 * kBM) * cdiv(op.n_extent, PairConfig::BN);
  const long long want = tiles < max_pairs ? tiles * (args.tail_split > 1 ? args.tail_split : 1) : tiles;
  const int pairs = (int)(want < max_pairs ? want : max_pairs);
  if (pairs <= 0) return DELS_OK;
  if (g_pair_kgroup == 2) {
    DELS_CHECK_PDL("tc_scorer_pair_kernel launch", launch_pdl(tc_scorer_pair_kernel<VB, STORE, 2>,
        dim3(2 * pairs), dim3(kTcThreads), PairConfig::kSmemBytes, st, ma0, mb0, ma1, mb1, mb0t, mb1t, args));
  } else {
    DELS_CHECK_PDL("tc_scorer_pair_kernel launch", launch_pdl(tc_scorer_pair_kernel<VB, STORE, 1>,
        dim3(2 * pairs), dim3(kTcThreads), PairConfig::kSmemBytes, st, ma0, mb0, ma1, mb1, mb0t, mb1t, args));
  }
  return DELS_OK;
}

TcArgs blank_args() {
  TcArgs a;
  std::memset(&a, 0, sizeof(a));
  a.k_splits = 1;
  a.n_pos = 1;
  a.group_m = 1;
  a.tail_split = 1;
  return a;
}

// Split-K plan of a projection GEMM [rows, K] x [n, K]^T.
struct SplitPlan {
  int bn, splits, kb_per_split, ld_out;
};

SplitPlan plan_projection(int rows, int K, int n) {
  SplitPlan p;
  p.bn = n <= 32 ? 32 : (n <= 64 ? 64 : (n <= 128 ? 128 : 256));
  const int total_kb = cdiv(K, kBK);
  const int base_tiles = cdiv(rows, kBM) * cdiv(n, p.bn);
  int splits = cdiv(kTargetCtas, base_tiles);
  const int max_splits = total_kb / 4 > 1 ? total_kb / 4 : 1;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  p.kb_per_split = cdiv(total_kb, splits);
  p.splits = cdiv(total_kb, p.kb_per_split);
  p.ld_out = (n + 3) & ~3;
  return p;
}

size_t projection_partials_bytes(int rows, int K, int n) {
  const SplitPlan p = plan_projection(rows, K, n);
  return align256((size_t)p.splits * rows * p.ld_out * sizeof(float));
}

// partial[split][row][n] = x[row, k-slice] . w[n, k-slice]
int launch_projection(const void* x, long long ld_x, const void* w, long long ld_w, int rows, int K, int n,
                      float* partials, int* status, int sm_count, cudaStream_t st, SplitPlan* plan_out,
                      __nv_bfloat16* out_bf16 = nullptr, long long ld_bf16 = 0,
                      const __nv_bfloat16* bias_bf16 = nullptr, bool out_vec = false) {
  const SplitPlan p = plan_projection(rows, K, n);
  TcOperands op;
  op.a0 = x;
  op.lda0 = ld_x;
  op.b0 = w;
  op.ldb0 = ld_w;
  op.K0 = K;
  op.m_extent = rows;
  op.n_extent = n;
  TcArgs a = blank_args();
  a.m_rows = rows;
  a.n_cols = n;
  a.k_splits = p.splits;
  a.kb_per_split = p.kb_per_split;
  a.status = status;
  a.out = partials;
  a.ld_out = p.ld_out;
  a.split_stride = (long long)rows * p.ld_out;
  if (out_bf16 != nullptr) {
    if (p.splits != 1) return fail(DELS_ERR_UNSUPPORTED, "bf16 GEMM output needs a single K split");
    // a wide B operand (an LM head): row tiles sweep it in groups so that it streams from
    // HBM once per group, and the last partial wave is split along N like the scorer's
    a.group_m = kScorerGroupM;
    // 32-column units for the last partial wave (the epilogue's chunk width): with few
    // rows the GEMM streams B at HBM speed, so the wave's time follows its widest unit
    a.tail_split = p.bn / 32;
    a.out = nullptr;
    a.out_bf16 = out_bf16;
    a.ld_out = ld_bf16;
    a.bias_bf16 = bias_bf16;
    a.out_vec = out_vec ? 1 : 0;
  }
  if (plan_out) *plan_out = p;
  switch (p.bn) {
    case 32: return launch_tc<32, kStore, false>(op, a, sm_count, st);
    case 64: return launch_tc<64, kStore, false>(op, a, sm_count, st);
    case 128: return launch_tc<128, kStore, false>(op, a, sm_count, st);
    default: return launch_tc<256, kStore, false>(op, a, sm_count, st);
  }
}

int check_common_score_args(int rows, int V, long long v_begin, const float* beta, const float* prior, int n_pos,
                            const int* keys_present) {
  if (rows < 0) return fail(DELS_ERR_INVALID_ARG, "rows must be >= 0 (got %d)", rows);
  if (V <= 0) return fail(DELS_ERR_INVALID_ARG, "V must be > 0 (got %d)", V);
  if (v_begin < 0 || v_begin + (long long)V > 0xFFFFFFFFll)
    return fail(DELS_ERR_INVALID_ARG, "vocab range [%lld, %lld) exceeds the 32-bit index space", v_begin,
                v_begin + V);
  if (prior != nullptr && beta == nullptr) return fail(DELS_ERR_INVALID_ARG, "beta is NULL but prior is given");
  if (n_pos <= 0) return fail(DELS_ERR_INVALID_ARG, "n_pos must be > 0 (got %d)", n_pos);
  if (prior != nullptr && !aligned16(prior)) return fail(DELS_ERR_ALIGNMENT, "prior must be 16-byte aligned");
  if (keys_present != nullptr && *keys_present == 0) return fail(DELS_ERR_INVALID_ARG, "keys is NULL");
  return DELS_OK;
}

int fused_argmax_common(const void* h, long long ld_h, const void* W, long long ld_w, const void* base,
                        long long ld_base, const void* s_scaled, long long ld_s, const void* Vr, long long ld_vr,
                        const float* prior, const float* beta, int n_pos, const int32_t* row_pos, int rows,
                        const int32_t* rows_dev, int H, int r, int V, long long v_begin, uint32_t flags,
                        int64_t* keys, int64_t* idx_out, float* score_out, void* ws, size_t ws_bytes,
                        cudaStream_t st, const TcArgs* gh = nullptr) {
  const int have_keys = keys != nullptr;
  int rc = check_common_score_args(rows, V, v_begin, beta, prior, n_pos, &have_keys);
  if (rc != DELS_OK) return rc;
  if (H < 0 || r < 0 || (H == 0 && r == 0 && base == nullptr))
    return fail(DELS_ERR_INVALID_ARG, "need H > 0 or r > 0 (H=%d, r=%d)", H, r);
  if (H > 0) {
    if ((rc = check_bf16_matrix("h", h, ld_h, H)) != DELS_OK) return rc;
    if ((rc = check_bf16_matrix("W", W, ld_w, H)) != DELS_OK) return rc;
  }
  if (r > 0) {
    if ((rc = check_bf16_matrix("s_scaled", s_scaled, ld_s, r)) != DELS_OK) return rc;
    if ((rc = check_bf16_matrix("Vr", Vr, ld_vr, r)) != DELS_OK) return rc;
  }
  if (idx_out == nullptr && score_out != nullptr)
    return fail(DELS_ERR_INVALID_ARG, "score_out needs idx_out (use dels_keys_decode for keys-only calls)");
  if (r == 0) return fail(DELS_ERR_UNSUPPORTED, "r must be > 0");
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, DELS_WS_HEADER_BYTES, &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (rows == 0) return DELS_OK;

  if ((flags & DELS_FLAG_KEYS_READY) == 0u) {
    DELS_CHECK_PDL("keys_init_kernel launch", launch_pdl(keys_init_kernel,
        dim3(cdiv(rows, 256) < 1024 ? cdiv(rows, 256) : 1024), dim3(256), 0, st,
        reinterpret_cast<long long*>(keys), rows, hdr.counter));
  }

  TcOperands op;
  op.a0 = h;
  op.lda0 = ld_h;
  op.b0 = W;
  op.ldb0 = ld_w;
  op.K0 = H;
  op.a1 = s_scaled;
  op.lda1 = ld_s;
  op.b1 = Vr;
  op.ldb1 = ld_vr;
  op.K1 = r;
  op.m_extent = rows;
  op.n_extent = V;
  TcArgs a = blank_args();
  a.m_rows = rows;
  a.m_rows_dev = rows_dev;
  a.n_cols = V;
  a.k_splits = 1;
  a.kb_per_split = cdiv(H, kBK) + cdiv(r, kBK);
  a.group_m = kScorerGroupM;
  a.tail_split = kScorerTailSplit;
  a.status = hdr.status;
  a.v_begin = v_begin;
  a.prior = prior;
  a.beta = beta;
  a.row_pos = row_pos;
  a.n_pos = n_pos;
  a.base = reinterpret_cast<const __nv_bfloat16*>(base);
  a.ld_base = ld_base;
  a.keys = reinterpret_cast<long long*>(keys);
  a.idx_out = reinterpret_cast<long long*>(idx_out);
  a.score_out = score_out;
  a.counter = hdr.counter;
  const bool vec_base = base != nullptr && aligned16(base) && (ld_base % 8) == 0;
  if (gh != nullptr) {
    // the next step's W_hh h on the plain skinny scorer's helper warps
    if (!(rows <= kSkinnyGhRows && g_use_skinny))
      return fail(DELS_ERR_UNSUPPORTED, "the fused gh projection needs at most %d rows and the skinny scorer",
                  kSkinnyGhRows);
    a.gh_w = gh->gh_w;
    a.gh_bias = gh->gh_bias;
    a.gh_x = gh->gh_x;
    a.gh_out = gh->gh_out;
    a.gh_rows = gh->gh_rows;
    a.gh_k = gh->gh_k;
    a.gh_b = rows;
    return launch_skinny<16, false, true>(op, a, ds->sm_count, st);
  }
  if (rows <= kSkinnyMaxRows && g_use_skinny) {
    // Decode-shaped call: the vocab tile is the MMA's M side, the rows its N side.  Above
    // kSkinnyStageRows rows the producer stages the epilogue operands (base logits when
    // TMA can address them, prior).
    const bool stage = rows > kSkinnyStageRows && (base == nullptr || vec_base);
    if (rows <= 16)
      return stage ? launch_skinny<16, true>(op, a, ds->sm_count, st) : launch_skinny<16, false>(op, a, ds->sm_count, st);
    return stage ? launch_skinny<32, true>(op, a, ds->sm_count, st) : launch_skinny<32, false>(op, a, ds->sm_count, st);
  }
  if (rows > kBM && ds->max_pairs > 0 && g_use_pairs) {
    // More than one 128-row tile: CTA pairs share each LM-head tile across two SMs.
    a.group_m = kScorerGroupM / 2;
    if (vec_base) return launch_scorer_pair<true>(op, a, ds->max_pairs, st);
    return launch_scorer_pair<false>(op, a, ds->max_pairs, st);
  }
  if (vec_base) return launch_tc<256, kArgmax, true>(op, a, ds->sm_count, st);
  return launch_tc<256, kArgmax, false>(op, a, ds->sm_count, st);
}

}  // namespace

// ======================================================================== C ABI
extern "C" {

int dels_version(void) { return kVersion; }

const char* dels_status_string(int status) {
  switch (status) {
    case DELS_OK: return "ok";
    case DELS_ERR_INVALID_ARG: return "invalid argument";
    case DELS_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case DELS_ERR_WORKSPACE: return "workspace missing or too small";
    case DELS_ERR_CUDA: return "CUDA error";
    case DELS_ERR_UNSUPPORTED: return "unsupported configuration";
    case DELS_ERR_DEVICE_TIMEOUT: return "a device-side wait timed out";
    default: return "unknown status";
  }
}

const char* dels_last_error(void) { return g_last_error.c_str(); }

int dels_init(int device) { return init_device(device); }

int dels_sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return fail(DELS_ERR_INVALID_ARG, "device out of range");
  int rc = init_device(device);
  if (rc != DELS_OK) return rc;
  return g_dev[device].sm_count;
}

size_t dels_rank_workspace_bytes(int rows, int K, int r) {
  if (rows <= 0 || K <= 0 || r <= 0) return DELS_WS_HEADER_BYTES;
  return DELS_WS_HEADER_BYTES + projection_partials_bytes(rows, K, r);
}

int dels_rank_project_bf16(const void* x, int64_t ld_x, const void* w_rank, int64_t ld_w, int rows, int K, int r,
                           int activation, const float* alpha, int n_pos, const int32_t* row_pos, void* s_out,
                           void* s_scaled, int64_t* keys, void* ws, size_t ws_bytes, void* stream) {
  int rc;
  if (rows < 0 || K <= 0 || r <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape rows=%d K=%d r=%d", rows, K, r);
  if (activation != DELS_ACT_IDENTITY && activation != DELS_ACT_SILU)
    return fail(DELS_ERR_INVALID_ARG, "unsupported rank activation %d", activation);
  if (n_pos <= 0) return fail(DELS_ERR_INVALID_ARG, "n_pos must be > 0");
  if (s_scaled == nullptr) return fail(DELS_ERR_INVALID_ARG, "s_scaled is NULL");
  if ((rc = check_bf16_matrix("x", x, ld_x, K)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w_rank", w_rank, ld_w, K)) != DELS_OK) return rc;
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, dels_rank_workspace_bytes(rows, K, r), &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (rows == 0) return DELS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + DELS_WS_HEADER_BYTES);
  SplitPlan plan;
  if ((rc = launch_projection(x, ld_x, w_rank, ld_w, rows, K, r, partials, hdr.status, ds->sm_count, st, &plan)) !=
      DELS_OK)
    return rc;
  const long long total = (long long)rows * r;
  const int grid = (int)(cdiv(total, 256) < 4 * ds->sm_count ? cdiv(total, 256) : 4 * ds->sm_count);
  DELS_CHECK_PDL("rank_finalize_kernel launch", launch_pdl(rank_finalize_kernel, dim3(grid), dim3(256), 0, st,
      partials, plan.splits, (long long)rows * plan.ld_out, plan.ld_out, rows, r, activation, alpha, n_pos,
      row_pos, reinterpret_cast<__nv_bfloat16*>(s_out), reinterpret_cast<__nv_bfloat16*>(s_scaled),
      reinterpret_cast<long long*>(keys), hdr.counter));
  return DELS_OK;
}

int dels_fused_argmax_bf16(const void* h, int64_t ld_h, const void* W, int64_t ld_w, const void* s_scaled,
                           int64_t ld_s, const void* Vr, int64_t ld_vr, const float* prior, const float* beta,
                           int n_pos, const int32_t* row_pos, int rows, const int32_t* rows_dev, int H, int r,
                           int V, int64_t v_begin, uint32_t flags, int64_t* keys, int64_t* idx_out,
                           float* score_out, void* ws, size_t ws_bytes, void* stream) {
  if (H <= 0) return fail(DELS_ERR_INVALID_ARG, "H must be > 0 (use dels_fused_argmax_base_bf16 without W.h)");
  return fused_argmax_common(h, ld_h, W, ld_w, nullptr, 0, s_scaled, ld_s, Vr, ld_vr, prior, beta, n_pos, row_pos,
                             rows, rows_dev, H, r, V, v_begin, flags, keys, idx_out, score_out, ws, ws_bytes,
                             reinterpret_cast<cudaStream_t>(stream));
}

int dels_fused_argmax_base_bf16(const void* base, int64_t ld_base, const void* s_scaled, int64_t ld_s,
                                const void* Vr, int64_t ld_vr, const float* prior, const float* beta, int n_pos,
                                const int32_t* row_pos, int rows, const int32_t* rows_dev, int r, int V,
                                int64_t v_begin, uint32_t flags, int64_t* keys, int64_t* idx_out,
                                float* score_out, void* ws, size_t ws_bytes, void* stream) {
  if (base == nullptr) return fail(DELS_ERR_INVALID_ARG, "base is NULL");
  if (ld_base < V) return fail(DELS_ERR_INVALID_ARG, "ld_base %lld < V %d", (long long)ld_base, V);
  if (r <= 0) return fail(DELS_ERR_INVALID_ARG, "r must be > 0");
  return fused_argmax_common(nullptr, 0, nullptr, 0, base, ld_base, s_scaled, ld_s, Vr, ld_vr, prior, beta, n_pos,
                             row_pos, rows, rows_dev, 0, r, V, v_begin, flags, keys, idx_out, score_out, ws,
                             ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int dels_fused_argmax_base_gru_bf16(const void* base, int64_t ld_base, const void* s_scaled, int64_t ld_s,
                                    const void* Vr, int64_t ld_vr, const float* prior, const float* beta, int n_pos,
                                    int rows, int r, int V, uint32_t flags, int64_t* keys, int64_t* idx_out,
                                    void* ws, size_t ws_bytes, const void* w_hh, const void* b_hh, const void* h,
                                    int G, void* gh_out, void* stream) {
  if (base == nullptr) return fail(DELS_ERR_INVALID_ARG, "base is NULL");
  if (ld_base < V) return fail(DELS_ERR_INVALID_ARG, "ld_base %lld < V %d", (long long)ld_base, V);
  if (r <= 0) return fail(DELS_ERR_INVALID_ARG, "r must be > 0");
  if (w_hh == nullptr || h == nullptr || gh_out == nullptr) return fail(DELS_ERR_INVALID_ARG, "NULL GRU operand");
  if (G <= 0 || (G % 8) != 0 || !aligned16(w_hh) || !aligned16(h))
    return fail(DELS_ERR_ALIGNMENT, "GRU hidden size %d must be a multiple of 8, w_hh and h 16-byte aligned", G);
  if (rows > kSkinnyGhRows) return fail(DELS_ERR_UNSUPPORTED, "at most %d rows (got %d)", kSkinnyGhRows, rows);
  TcArgs gh;
  std::memset(&gh, 0, sizeof(gh));
  gh.gh_w = reinterpret_cast<const __nv_bfloat16*>(w_hh);
  gh.gh_bias = reinterpret_cast<const __nv_bfloat16*>(b_hh);
  gh.gh_x = reinterpret_cast<const __nv_bfloat16*>(h);
  gh.gh_out = reinterpret_cast<__nv_bfloat16*>(gh_out);
  gh.gh_rows = 3 * G;
  gh.gh_k = G;
  return fused_argmax_common(nullptr, 0, nullptr, 0, base, ld_base, s_scaled, ld_s, Vr, ld_vr, prior, beta, n_pos,
                             nullptr, rows, nullptr, 0, r, V, 0, flags, keys, idx_out, nullptr, ws, ws_bytes,
                             reinterpret_cast<cudaStream_t>(stream), &gh);
}

size_t dels_score_workspace_bytes(int rows, int H, int r) {
  if (rows <= 0 || H <= 0 || r <= 0) return DELS_WS_HEADER_BYTES;
  return DELS_WS_HEADER_BYTES + align256((size_t)rows * 8) + align256((size_t)rows * r * 2) +
         projection_partials_bytes(rows, H, r);
}

int dels_draft_score_bf16(const void* h, int64_t ld_h, const void* W, int64_t ld_w, const void* w_rank,
                          int64_t ld_wr, const void* Vr, int64_t ld_vr, const float* prior, const float* alpha,
                          const float* beta, int n_pos, const int32_t* row_pos, int rows, const int32_t* rows_dev,
                          int H, int r, int V, int64_t v_begin, int activation, int64_t* keys, int64_t* idx_out,
                          float* score_out, void* ws, size_t ws_bytes, void* stream) {
  int rc;
  if (rows < 0 || H <= 0 || r <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape rows=%d H=%d r=%d", rows, H, r);
  const size_t need = dels_score_workspace_bytes(rows, H, r);
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, need, &hdr)) != DELS_OK) return rc;
  if (rows == 0) return DELS_OK;
  char* base = reinterpret_cast<char*>(ws);
  int64_t* ws_keys = reinterpret_cast<int64_t*>(base + DELS_WS_HEADER_BYTES);
  void* s_scaled = base + DELS_WS_HEADER_BYTES + align256((size_t)rows * 8);
  // The rank projection's partials live after s_scaled; hand it a view of the
  // workspace whose header is shared with this call.
  const size_t part_off = DELS_WS_HEADER_BYTES + align256((size_t)rows * 8) + align256((size_t)rows * r * 2);
  if (keys == nullptr) keys = ws_keys;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((rc = check_bf16_matrix("h", h, ld_h, H)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w_rank", w_rank, ld_wr, H)) != DELS_OK) return rc;
  if (activation != DELS_ACT_IDENTITY && activation != DELS_ACT_SILU)
    return fail(DELS_ERR_INVALID_ARG, "unsupported rank activation %d", activation);
  const int have_keys = 1;
  if ((rc = check_common_score_args(rows, V, v_begin, beta, prior, n_pos, &have_keys)) != DELS_OK) return rc;
  float* partials = reinterpret_cast<float*>(base + part_off);
  SplitPlan plan;
  if ((rc = launch_projection(h, ld_h, w_rank, ld_wr, rows, H, r, partials, hdr.status, ds->sm_count, st, &plan)) !=
      DELS_OK)
    return rc;
  const long long total = (long long)rows * r;
  const int grid = (int)(cdiv(total, 256) < 4 * ds->sm_count ? cdiv(total, 256) : 4 * ds->sm_count);
  DELS_CHECK_PDL("rank_finalize_kernel launch", launch_pdl(rank_finalize_kernel, dim3(grid), dim3(256), 0, st,
      partials, plan.splits, (long long)rows * plan.ld_out, plan.ld_out, rows, r, activation, alpha, n_pos,
      row_pos, nullptr, reinterpret_cast<__nv_bfloat16*>(s_scaled), reinterpret_cast<long long*>(keys),
      hdr.counter));
  return fused_argmax_common(h, ld_h, W, ld_w, nullptr, 0, s_scaled, r, Vr, ld_vr, prior, beta, n_pos, row_pos,
                             rows, rows_dev, H, r, V, v_begin, DELS_FLAG_KEYS_READY, keys, idx_out, score_out, ws,
                             ws_bytes, st);
}

size_t dels_score_f32_workspace_bytes(int rows, int H, int r) {
  if (rows <= 0 || H <= 0 || r <= 0) return DELS_WS_HEADER_BYTES;
  // keys, s' = alpha * s, and one pass's rows transposed ([H][16] and [r][16])
  return DELS_WS_HEADER_BYTES + align256((size_t)rows * 8) + align256((size_t)rows * r * 4) +
         align256((size_t)H * 16 * 4) + align256((size_t)r * 16 * 4);
}

int dels_draft_score_f32(const float* h, int64_t ld_h, const float* W, int64_t ld_w, const float* w_rank,
                         int64_t ld_wr, const float* Vr, int64_t ld_vr, const float* prior, const float* alpha,
                         const float* beta, int n_pos, const int32_t* row_pos, int rows, int H, int r, int V,
                         int64_t v_begin, int64_t* keys, int64_t* idx_out, float* score_out, void* ws,
                         size_t ws_bytes, void* stream) {
  int rc;
  if (rows < 0 || H <= 0 || r <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape rows=%d H=%d r=%d", rows, H, r);
  if ((H % 4) != 0 || (r % 4) != 0)
    return fail(DELS_ERR_UNSUPPORTED, "fp32 scorer needs H %% 4 == 0 and r %% 4 == 0 (H=%d, r=%d)", H, r);
  if (h == nullptr || W == nullptr || w_rank == nullptr || Vr == nullptr)
    return fail(DELS_ERR_INVALID_ARG, "NULL operand");
  if (!aligned16(W) || !aligned16(Vr) || !aligned16(h) || (ld_w % 4) != 0 || (ld_vr % 4) != 0 || (ld_h % 4) != 0 ||
      ld_w < H || ld_vr < r || ld_h < H || ld_wr < H)
    return fail(DELS_ERR_ALIGNMENT, "fp32 h / W / Vr need 16-byte aligned rows (ld %% 4 == 0)");
  const int have_keys = 1;
  if ((rc = check_common_score_args(rows, V, v_begin, beta, prior, n_pos, &have_keys)) != DELS_OK) return rc;
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, dels_score_f32_workspace_bytes(rows, H, r), &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (rows == 0) return DELS_OK;
  if (idx_out == nullptr && score_out != nullptr)
    return fail(DELS_ERR_INVALID_ARG, "score_out needs idx_out (use dels_keys_decode for keys-only calls)");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* base = reinterpret_cast<char*>(ws);
  if (keys == nullptr) keys = reinterpret_cast<int64_t*>(base + DELS_WS_HEADER_BYTES);
  float* s_scaled = reinterpret_cast<float*>(base + DELS_WS_HEADER_BYTES + align256((size_t)rows * 8));
  float* hT = reinterpret_cast<float*>(reinterpret_cast<char*>(s_scaled) + align256((size_t)rows * r * 4));
  float* sT = reinterpret_cast<float*>(reinterpret_cast<char*>(hT) + align256((size_t)H * 16 * 4));

  {
    const int warps = rows * r;
    const int grid = cdiv(warps, 8) < 8 * ds->sm_count ? cdiv(warps, 8) : 8 * ds->sm_count;
    f32_rank_kernel<<<grid, 256, 0, st>>>(h, ld_h, w_rank, ld_wr, rows, H, r, alpha, n_pos, row_pos, s_scaled,
                                          reinterpret_cast<long long*>(keys), hdr.counter);
    DELS_CHECK_LAUNCH("f32_rank_kernel launch");
  }
  if ((rc = ensure_encode()) != DELS_OK) return rc;
  // W / Vr: 32-float boxes of one vocabulary tile, 128-byte swizzle (the kernel reads 32
  // rows at one k)
  CUtensorMap mw, mvr;
  if ((rc = make_map_f32(&mw, W, H, V, ld_w, f32_score_tile_rows(), true)) != DELS_OK) return rc;
  if ((rc = make_map_f32(&mvr, Vr, r, V, ld_vr, f32_score_tile_rows(), true)) != DELS_OK) return rc;
  const int kb0 = cdiv(H, 64), kb1 = cdiv(r, 64);
  // the transposed pass buffers: [k][16] rows, 32 k per box
  CUtensorMap mh, ms;
  if ((rc = make_map_f32(&mh, hT, 16, H, 16, 32, false, 16)) != DELS_OK) return rc;
  if ((rc = make_map_f32(&ms, sT, 16, r, 16, 32, false, 16)) != DELS_OK) return rc;
  for (int row0 = 0; row0 < rows; row0 += 16) {
    const int nrows = rows - row0 < 16 ? rows - row0 : 16;
    {
      const long long total = (long long)(H + r) * 16;
      const int grid = (int)(cdiv(total, 256) < 2 * ds->sm_count ? cdiv(total, 256) : 2 * ds->sm_count);
      f32_transpose_pass_kernel<<<grid, 256, 0, st>>>(h + (long long)row0 * ld_h, ld_h, H,
                                                      s_scaled + (long long)row0 * r, r, r, nrows, hT, sT);
      DELS_CHECK_LAUNCH("f32_transpose_pass_kernel launch");
    }
    cudaError_t e = f32_score_launch(ds->sm_count, st, mw, mh, mvr, ms, kb0, kb1, prior, beta, n_pos, row_pos, row0,
                                     nrows, V, v_begin, reinterpret_cast<long long*>(keys), hdr.status);
    if (e != cudaSuccess) return cuda_fail(e, "f32_score_kernel launch");
  }
  if (idx_out != nullptr) {
    DELS_CHECK_PDL("keys_decode_kernel launch", launch_pdl(keys_decode_kernel, dim3(cdiv(rows, 256)),
        dim3(256), 0, st, reinterpret_cast<const long long*>(keys), rows, nullptr,
        reinterpret_cast<long long*>(idx_out), score_out));
  }
  return DELS_OK;
}

int dels_keys_init(int64_t* keys, int rows, void* ws, void* stream) {
  if (keys == nullptr || rows < 0) return fail(DELS_ERR_INVALID_ARG, "keys NULL or rows < 0");
  unsigned* counter = nullptr;
  if (ws != nullptr) {
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(DELS_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
    counter = reinterpret_cast<unsigned*>(ws);
  }
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (rows == 0 && counter == nullptr) return DELS_OK;
  const int grid = rows > 0 ? (cdiv(rows, 256) < 1024 ? cdiv(rows, 256) : 1024) : 1;
  DELS_CHECK_PDL("keys_init_kernel launch", launch_pdl(keys_init_kernel, dim3(grid), dim3(256), 0,
      reinterpret_cast<cudaStream_t>(stream), reinterpret_cast<long long*>(keys), rows, counter));
  return DELS_OK;
}

int dels_keys_decode(const int64_t* keys, int rows, const int32_t* rows_dev, int64_t* idx_out, float* score_out,
                     void* stream) {
  if (keys == nullptr || rows < 0) return fail(DELS_ERR_INVALID_ARG, "keys NULL or rows < 0");
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (rows == 0) return DELS_OK;
  const int grid = cdiv(rows, 256) < 1024 ? cdiv(rows, 256) : 1024;
  DELS_CHECK_PDL("keys_decode_kernel launch", launch_pdl(keys_decode_kernel, dim3(grid), dim3(256), 0,
      reinterpret_cast<cudaStream_t>(stream), reinterpret_cast<const long long*>(keys), rows, rows_dev,
      reinterpret_cast<long long*>(idx_out), score_out));
  return DELS_OK;
}

int dels_accept_offsets(const int64_t* draft, int64_t ld_draft, const int64_t* target, int64_t ld_target,
                        int n_seq, int n_draft, int commit_extra, int32_t* accept, int32_t* offsets, void* stream) {
  if (n_seq < 0 || n_draft < 0) return fail(DELS_ERR_INVALID_ARG, "n_seq and n_draft must be >= 0");
  if (commit_extra != 0 && commit_extra != 1) return fail(DELS_ERR_INVALID_ARG, "commit_extra must be 0 or 1");
  if (offsets == nullptr || (n_seq > 0 && accept == nullptr))
    return fail(DELS_ERR_INVALID_ARG, "accept / offsets is NULL");
  if (n_seq > 0 && n_draft > 0 && (draft == nullptr || target == nullptr))
    return fail(DELS_ERR_INVALID_ARG, "draft / target is NULL");
  if (ld_draft < n_draft || ld_target < n_draft)
    return fail(DELS_ERR_INVALID_ARG, "leading dimensions must be >= n_draft");
  if ((long long)n_seq * (n_draft + commit_extra) > 0x7FFFFFFFll)
    return fail(DELS_ERR_INVALID_ARG, "packed row count overflows int32");
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  accept_offsets_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const long long*>(draft), ld_draft, reinterpret_cast<const long long*>(target), ld_target,
      n_seq, n_draft, commit_extra, accept, offsets);
  DELS_CHECK_LAUNCH("accept_offsets_kernel launch");
  return DELS_OK;
}

int dels_pack_rows_bf16(const void* hidden, int64_t ld_seq, int64_t ld_row, int n_seq, int P, int H,
                        const int32_t* accept, const int32_t* offsets, void* packed, int64_t ld_packed,
                        int32_t* row_pos, void* stream) {
  if (n_seq < 0 || P <= 0 || H <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape n_seq=%d P=%d H=%d", n_seq, P, H);
  if (hidden == nullptr || accept == nullptr || offsets == nullptr || packed == nullptr)
    return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (ld_row < H || ld_seq < (long long)P * ld_row - (ld_row - H) || ld_packed < H)
    return fail(DELS_ERR_INVALID_ARG, "inconsistent strides");
  if ((long long)n_seq * P > 0x7FFFFFFFll) return fail(DELS_ERR_INVALID_ARG, "too many rows");
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (n_seq == 0) return DELS_OK;
  pack_rows_kernel<<<n_seq * P, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(hidden), ld_seq, ld_row, n_seq, P, H, accept, offsets,
      reinterpret_cast<__nv_bfloat16*>(packed), ld_packed, row_pos);
  DELS_CHECK_LAUNCH("pack_rows_kernel launch");
  return DELS_OK;
}

int dels_selftest_bounded_wait(int* status, uint64_t* waited_ns, double limit_ms, void* stream) {
  if (status == nullptr || waited_ns == nullptr) return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (!(limit_ms > 0.0 && limit_ms <= 1000.0)) return fail(DELS_ERR_INVALID_ARG, "limit_ms must be in (0, 1000]");
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  wait_selftest_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      status, (unsigned long long)(limit_ms * 1e6), reinterpret_cast<unsigned long long*>(waited_ns));
  DELS_CHECK_LAUNCH("wait_selftest_kernel launch");
  return DELS_OK;
}


size_t dels_rnn_workspace_bytes(int n_seq, int T, int H, int r) {
  if (n_seq <= 0 || T <= 0 || H <= 0 || r <= 0) return DELS_WS_HEADER_BYTES;
  return DELS_WS_HEADER_BYTES + projection_partials_bytes(n_seq * T, H, r);
}

int dels_rnn_rank_states_bf16(const void* x, int64_t ld_x, const void* w_in, int64_t ld_win, const void* w_s,
                              const float* bias, const float* alpha, int n_seq, int T, int H, int r,
                              void* s_scaled, void* s_out, int64_t* keys, void* ws, size_t ws_bytes,
                              void* stream) {
  int rc;
  if (n_seq < 0 || T <= 0 || H <= 0 || r <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape");
  if (r > 256 || (r % 2) != 0) return fail(DELS_ERR_UNSUPPORTED, "RNN rank r must be even and <= 256 (got %d)", r);
  if (w_s == nullptr || s_scaled == nullptr) return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if ((long long)n_seq * T > 0x7FFFFFFFll) return fail(DELS_ERR_INVALID_ARG, "too many rows");
  if ((rc = check_bf16_matrix("x", x, ld_x, H)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w_in", w_in, ld_win, H)) != DELS_OK) return rc;
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, dels_rnn_workspace_bytes(n_seq, T, H, r), &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (n_seq == 0) return DELS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int rows = n_seq * T;
  float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + DELS_WS_HEADER_BYTES);
  SplitPlan plan;
  if ((rc = launch_projection(x, ld_x, w_in, ld_win, rows, H, r, partials, hdr.status, ds->sm_count, st, &plan)) !=
      DELS_OK)
    return rc;
  rnn_recurrence_kernel<<<cdiv(n_seq, kRnnSeqs), 256, rnn_smem_bytes(r), st>>>(
      partials, plan.splits, (long long)rows * plan.ld_out, plan.ld_out,
      reinterpret_cast<const __nv_bfloat16*>(w_s), bias, alpha, n_seq, T, r,
      reinterpret_cast<__nv_bfloat16*>(s_scaled), reinterpret_cast<__nv_bfloat16*>(s_out),
      reinterpret_cast<long long*>(keys), hdr.counter);
  DELS_CHECK_LAUNCH("rnn_recurrence_kernel launch");
  return DELS_OK;
}

int dels_gru_step_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table, int64_t ld_table,
                       const void* w_hh, const void* b_hh, const void* h_in, void* h_out, int B, int G, int V,
                       void* ws, void* stream) {
  if (B < 0 || G <= 0 || V <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape B=%d G=%d V=%d", B, G, V);
  if ((G % 8) != 0) return fail(DELS_ERR_UNSUPPORTED, "GRU hidden size %d must be a multiple of 8", G);
  if (tokens == nullptr || gi_table == nullptr || w_hh == nullptr || h_out == nullptr)
    return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (!aligned16(w_hh) || (h_in != nullptr && !aligned16(h_in)) || !aligned16(h_out))
    return fail(DELS_ERR_ALIGNMENT, "w_hh / h_in / h_out must be 16-byte aligned");
  if (ld_table < 3LL * G) return fail(DELS_ERR_INVALID_ARG, "gi table leading dimension < 3G");
  if (gru_smem_bytes(G) > (size_t)kMaxSmem) return fail(DELS_ERR_UNSUPPORTED, "GRU hidden size %d too large", G);
  int* status = ws != nullptr ? reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + 4) : nullptr;
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (B == 0) return DELS_OK;
  const int rows_per_pass = runner_rows_per_pass(B);
  DELS_CHECK_PDL("gru_step_kernel launch", launch_pdl(gru_step_kernel_for(rows_per_pass), dim3(cdiv(G, kGruCols)),
      dim3(kGruThreads), gru_smem_bytes(G, rows_per_pass), reinterpret_cast<cudaStream_t>(stream),
      reinterpret_cast<const long long*>(tokens), tok_stride, token_keys,
      reinterpret_cast<const __nv_bfloat16*>(gi_table), ld_table,
      reinterpret_cast<const __nv_bfloat16*>(w_hh), reinterpret_cast<const __nv_bfloat16*>(b_hh),
      reinterpret_cast<const __nv_bfloat16*>(h_in), reinterpret_cast<__nv_bfloat16*>(h_out), B, G, V,
      status));
  return DELS_OK;
}

int dels_gru_gates_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                        int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in, void* h_out, int B, int G,
                        int V, void* ws, void* stream) {
  if (B < 0 || G <= 0 || V <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape B=%d G=%d V=%d", B, G, V);
  if (tokens == nullptr || gi_table == nullptr || gh == nullptr || h_out == nullptr)
    return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (ld_table < 3LL * G) return fail(DELS_ERR_INVALID_ARG, "gi table leading dimension < 3G");
  if (ld_gh < 3LL * G) return fail(DELS_ERR_INVALID_ARG, "gh leading dimension < 3G");
  int* status = ws != nullptr ? reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + 4) : nullptr;
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (B == 0) return DELS_OK;
  const long long total = (long long)B * G;
  const int grid = (int)(cdiv(total, 256) < 4 * ds->sm_count ? cdiv(total, 256) : 4 * ds->sm_count);
  DELS_CHECK_PDL("gru_gates_kernel launch", launch_pdl(gru_gates_kernel, dim3(grid), dim3(256), 0,
      reinterpret_cast<cudaStream_t>(stream), reinterpret_cast<const long long*>(tokens), tok_stride, token_keys,
      reinterpret_cast<const __nv_bfloat16*>(gi_table), ld_table, reinterpret_cast<const __nv_bfloat16*>(gh),
      (long long)ld_gh, reinterpret_cast<const __nv_bfloat16*>(h_in), reinterpret_cast<__nv_bfloat16*>(h_out), B, G,
      V, status));
  return DELS_OK;
}

static int rank_gemv_common(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias,
                            const void* addend, int64_t ld_add, int B, int K, int r, int activation,
                            const float* alpha, int n_pos, const int32_t* row_pos, void* s_out, void* s_scaled,
                            int64_t* keys, void* ws, void* stream, const GruGateSrc* gate = nullptr) {
  int rc;
  if (B < 0 || K <= 0 || r <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape B=%d K=%d r=%d", B, K, r);
  if ((K % 8) != 0) return fail(DELS_ERR_UNSUPPORTED, "K = %d must be a multiple of 8", K);
  if (activation != DELS_ACT_IDENTITY && activation != DELS_ACT_SILU)
    return fail(DELS_ERR_INVALID_ARG, "unsupported rank activation %d", activation);
  if (n_pos <= 0 || s_scaled == nullptr) return fail(DELS_ERR_INVALID_ARG, "n_pos <= 0 or s_scaled NULL");
  if (gate == nullptr && (rc = check_bf16_matrix("x", x, ld_x, K)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w_rank", w, ld_w, K)) != DELS_OK) return rc;
  if (addend != nullptr && ld_add < r) return fail(DELS_ERR_INVALID_ARG, "z leading dimension %lld < %d",
                                                   (long long)ld_add, r);
  if (rank_gemv_smem_bytes(K) > (size_t)kMaxSmem) return fail(DELS_ERR_UNSUPPORTED, "K = %d too large", K);
  unsigned* counter = ws != nullptr ? reinterpret_cast<unsigned*>(ws) : nullptr;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (B == 0) return DELS_OK;
  const int grid = cdiv(r, kGemvThreads / 32) < 2 * ds->sm_count ? cdiv(r, kGemvThreads / 32) : 2 * ds->sm_count;
  const int rows_per_pass = runner_rows_per_pass(B);
  DELS_CHECK_PDL("rank_gemv_kernel launch", launch_pdl(rank_gemv_kernel_for(rows_per_pass), dim3(grid),
      dim3(kGemvThreads), rank_gemv_smem_bytes(K, rows_per_pass), reinterpret_cast<cudaStream_t>(stream),
      reinterpret_cast<const __nv_bfloat16*>(x), ld_x, reinterpret_cast<const __nv_bfloat16*>(w), ld_w,
      reinterpret_cast<const __nv_bfloat16*>(bias), reinterpret_cast<const __nv_bfloat16*>(addend),
      (long long)ld_add, B, K, r, activation, alpha, n_pos, row_pos, reinterpret_cast<__nv_bfloat16*>(s_out),
      reinterpret_cast<__nv_bfloat16*>(s_scaled), reinterpret_cast<long long*>(keys), counter,
      gate != nullptr ? *gate : GruGateSrc{}));
  return DELS_OK;
}

int dels_rank_gemv_bf16(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias, int B, int K,
                        int r, int activation, const float* alpha, int n_pos, const int32_t* row_pos, void* s_out,
                        void* s_scaled, int64_t* keys, void* ws, void* stream) {
  return rank_gemv_common(x, ld_x, w, ld_w, bias, nullptr, 0, B, K, r, activation, alpha, n_pos, row_pos, s_out,
                          s_scaled, keys, ws, stream);
}

// The GRU gates of (tokens, gi_table, gh, h_in) as the x source of rank_gemv_common.
static int gru_gate_source(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                           int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in, void* h_out, int B,
                           int G, int V, void* ws, GruGateSrc* gate) {
  if (B < 0 || G <= 0 || V <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape B=%d G=%d V=%d", B, G, V);
  if (tokens == nullptr || gi_table == nullptr || gh == nullptr || h_out == nullptr)
    return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if ((G % 8) != 0 || (ld_table % 8) != 0 || (ld_gh % 8) != 0 || !aligned16(gi_table) || !aligned16(gh) ||
      !aligned16(h_out) || (h_in != nullptr && !aligned16(h_in)))
    return fail(DELS_ERR_ALIGNMENT, "gi table / gh / h rows must be 16-byte aligned (G, ld %% 8 == 0)");
  if (ld_table < 3LL * G || ld_gh < 3LL * G) return fail(DELS_ERR_INVALID_ARG, "gi / gh leading dimension < 3G");
  gate->tokens = reinterpret_cast<const long long*>(tokens);
  gate->tok_stride = tok_stride;
  gate->token_keys = token_keys != 0 ? 1 : 0;
  gate->table = reinterpret_cast<const __nv_bfloat16*>(gi_table);
  gate->ld_table = ld_table;
  gate->gh = reinterpret_cast<const __nv_bfloat16*>(gh);
  gate->ld_gh = ld_gh;
  gate->h_in = reinterpret_cast<const __nv_bfloat16*>(h_in);
  gate->h_out = reinterpret_cast<__nv_bfloat16*>(h_out);
  gate->V = V;
  gate->status = ws != nullptr ? reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + 4) : nullptr;
  return DELS_OK;
}

int dels_gru_rank_gemv_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                            int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in, void* h_out, int B,
                            int G, int V, const void* w_rank, int64_t ld_w, const void* bias, int r, int activation,
                            const float* alpha, void* s_scaled, int64_t* keys, void* ws, void* stream) {
  GruGateSrc gate;
  int rc = gru_gate_source(tokens, tok_stride, token_keys, gi_table, ld_table, gh, ld_gh, h_in, h_out, B, G, V, ws,
                           &gate);
  if (rc != DELS_OK) return rc;
  return rank_gemv_common(nullptr, G, w_rank, ld_w, bias, nullptr, 0, B, G, r, activation, alpha, 1, nullptr,
                          nullptr, s_scaled, keys, ws, stream, &gate);
}

int dels_gru_correction_mid_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                                 int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in, void* h_out,
                                 int B, int G, int V, const void* w_s, int64_t ld_ws, const void* z, int64_t ld_z,
                                 int M, const float* alpha, void* s_scaled, int64_t* keys, void* ws, void* stream) {
  if (z == nullptr) return fail(DELS_ERR_INVALID_ARG, "z is NULL");
  GruGateSrc gate;
  int rc = gru_gate_source(tokens, tok_stride, token_keys, gi_table, ld_table, gh, ld_gh, h_in, h_out, B, G, V, ws,
                           &gate);
  if (rc != DELS_OK) return rc;
  return rank_gemv_common(nullptr, G, w_s, ld_ws, nullptr, z, ld_z, B, G, M, DELS_ACT_IDENTITY, alpha, 1, nullptr,
                          nullptr, s_scaled, keys, ws, stream, &gate);
}

int dels_correction_mid_bf16(const void* h, int64_t ld_h, const void* w_s, int64_t ld_ws, const void* z,
                             int64_t ld_z, int B, int G, int M, const float* alpha, void* s_scaled, int64_t* keys,
                             void* ws, void* stream) {
  if (z == nullptr) return fail(DELS_ERR_INVALID_ARG, "z is NULL");
  return rank_gemv_common(h, ld_h, w_s, ld_ws, nullptr, z, ld_z, B, G, M, DELS_ACT_IDENTITY, alpha, 1, nullptr,
                          nullptr, s_scaled, keys, ws, stream);
}

size_t dels_linear_workspace_bytes(int rows, int K, int N) {
  if (rows <= 0 || K <= 0 || N <= 0) return DELS_WS_HEADER_BYTES;
  // one K split: the GEMM writes the bf16 result itself, no partial sums
  if (plan_projection(rows, K, N).splits == 1) return DELS_WS_HEADER_BYTES;
  return DELS_WS_HEADER_BYTES + projection_partials_bytes(rows, K, N);
}

int dels_linear_bf16(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias, int rows, int K,
                     int N, void* out, int64_t ld_out, void* ws, size_t ws_bytes, void* stream) {
  int rc;
  if (rows < 0 || K <= 0 || N <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape rows=%d K=%d N=%d", rows, K, N);
  if (out == nullptr || ld_out < N) return fail(DELS_ERR_INVALID_ARG, "out is NULL or ld_out < N");
  if ((rc = check_bf16_matrix("x", x, ld_x, K)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w", w, ld_w, K)) != DELS_OK) return rc;
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, dels_linear_workspace_bytes(rows, K, N), &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (rows == 0) return DELS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (plan_projection(rows, K, N).splits == 1) {
    // enough output tiles to fill the device without splitting K (vocabulary-sized N):
    // one launch, bf16 written by the GEMM's epilogue
    const bool vec = aligned16(out) && (ld_out % 8) == 0 && (bias == nullptr || aligned16(bias));
    if (rows > kBM && ds->max_pairs > 0 && g_use_pairs) {
      // more than one 128-row tile: CTA pairs (256-row tiles, each SM stages half of
      // every B tile), as the scorer does for the same shapes
      TcOperands op;
      op.a0 = x;
      op.lda0 = ld_x;
      op.b0 = w;
      op.ldb0 = ld_w;
      op.K0 = K;
      op.m_extent = rows;
      op.n_extent = N;
      TcArgs a = blank_args();
      a.m_rows = rows;
      a.n_cols = N;
      a.kb_per_split = cdiv(K, kBK);
      a.group_m = kScorerGroupM / 2;
      a.tail_split = kScorerTailSplit;
      a.status = hdr.status;
      a.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out);
      a.ld_out = ld_out;
      a.bias_bf16 = reinterpret_cast<const __nv_bfloat16*>(bias);
      a.out_vec = vec ? 1 : 0;
      return launch_scorer_pair<false, true>(op, a, ds->max_pairs, st);
    }
    return launch_projection(x, ld_x, w, ld_w, rows, K, N, nullptr, hdr.status, ds->sm_count, st, nullptr,
                             reinterpret_cast<__nv_bfloat16*>(out), ld_out,
                             reinterpret_cast<const __nv_bfloat16*>(bias), vec);
  }
  float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + DELS_WS_HEADER_BYTES);
  SplitPlan plan;
  if ((rc = launch_projection(x, ld_x, w, ld_w, rows, K, N, partials, hdr.status, ds->sm_count, st, &plan)) !=
      DELS_OK)
    return rc;
  const long long total = (long long)rows * N;
  const int grid = (int)(cdiv(total, 256) < 4 * ds->sm_count ? cdiv(total, 256) : 4 * ds->sm_count);
  DELS_CHECK_PDL("linear_finalize_kernel launch", launch_pdl(linear_finalize_kernel, dim3(grid), dim3(256), 0, st,
      partials, plan.splits, (long long)rows * plan.ld_out, (long long)plan.ld_out, rows, N,
      reinterpret_cast<const __nv_bfloat16*>(bias), reinterpret_cast<__nv_bfloat16*>(out), (long long)ld_out));
  return DELS_OK;
}

size_t dels_gru_step_tc_workspace_bytes(int B, int G) {
  if (B <= 0 || G <= 0) return DELS_WS_HEADER_BYTES;
  return DELS_WS_HEADER_BYTES + projection_partials_bytes(B, G, 3 * G);
}

int dels_gru_step_tc_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                          int64_t ld_table,
                          const void* w_hh, const void* b_hh, const void* h_in, void* h_out, int B, int G, int V,
                          void* ws, size_t ws_bytes, void* stream) {
  int rc;
  if (B < 0 || G <= 0 || V <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape B=%d G=%d V=%d", B, G, V);
  if (tokens == nullptr || gi_table == nullptr || h_in == nullptr || h_out == nullptr)
    return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (ld_table < 3LL * G) return fail(DELS_ERR_INVALID_ARG, "gi table leading dimension < 3G");
  if ((rc = check_bf16_matrix("h_in", h_in, G, G)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w_hh", w_hh, G, G)) != DELS_OK) return rc;
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, dels_gru_step_tc_workspace_bytes(B, G), &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (B == 0) return DELS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + DELS_WS_HEADER_BYTES);
  SplitPlan plan;
  if ((rc = launch_projection(h_in, G, w_hh, G, B, G, 3 * G, partials, hdr.status, ds->sm_count, st, &plan)) !=
      DELS_OK)
    return rc;
  const long long total = (long long)B * G;
  const int grid = (int)(cdiv(total, 256) < 4 * ds->sm_count ? cdiv(total, 256) : 4 * ds->sm_count);
  DELS_CHECK_PDL("gru_finalize_kernel launch", launch_pdl(gru_finalize_kernel, dim3(grid), dim3(256), 0, st,
      partials, plan.splits, (long long)B * plan.ld_out, (long long)plan.ld_out,
      reinterpret_cast<const long long*>(tokens), (long long)tok_stride, token_keys,
      reinterpret_cast<const __nv_bfloat16*>(gi_table), (long long)ld_table,
      reinterpret_cast<const __nv_bfloat16*>(b_hh), reinterpret_cast<const __nv_bfloat16*>(h_in),
      reinterpret_cast<__nv_bfloat16*>(h_out), B, G, V, hdr.status));
  return DELS_OK;
}

size_t dels_correction_mid_tc_workspace_bytes(int B, int G, int M) {
  // always split-K partials: the SiLU epilogue runs in the finalisation kernel
  if (B <= 0 || G <= 0 || M <= 0) return DELS_WS_HEADER_BYTES;
  return DELS_WS_HEADER_BYTES + projection_partials_bytes(B, G, M);
}

int dels_correction_mid_tc_bf16(const void* h, int64_t ld_h, const void* w_s, int64_t ld_ws, const void* z,
                                int64_t ld_z, int B, int G, int M, const float* alpha, void* s_scaled, int64_t* keys,
                                void* ws, size_t ws_bytes, void* stream) {
  int rc;
  if (B < 0 || G <= 0 || M <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape B=%d G=%d M=%d", B, G, M);
  if (z == nullptr || s_scaled == nullptr || alpha == nullptr) return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (ld_z < M) return fail(DELS_ERR_INVALID_ARG, "z leading dimension %lld < %d", (long long)ld_z, M);
  if ((rc = check_bf16_matrix("h", h, ld_h, G)) != DELS_OK) return rc;
  if ((rc = check_bf16_matrix("w_s", w_s, ld_ws, G)) != DELS_OK) return rc;
  WsHeader hdr;
  if ((rc = ws_header(ws, ws_bytes, dels_correction_mid_tc_workspace_bytes(B, G, M), &hdr)) != DELS_OK) return rc;
  DeviceState* ds = nullptr;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (B == 0) return DELS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + DELS_WS_HEADER_BYTES);
  SplitPlan plan;
  if ((rc = launch_projection(h, ld_h, w_s, ld_ws, B, G, M, partials, hdr.status, ds->sm_count, st, &plan)) !=
      DELS_OK)
    return rc;
  const long long total = (long long)B * M;
  const int grid = (int)(cdiv(total, 256) < 4 * ds->sm_count ? cdiv(total, 256) : 4 * ds->sm_count);
  DELS_CHECK_PDL("correction_finalize_kernel launch", launch_pdl(correction_finalize_kernel, dim3(grid), dim3(256),
      0, st, partials, plan.splits, (long long)B * plan.ld_out, (long long)plan.ld_out, B, M,
      reinterpret_cast<const __nv_bfloat16*>(z), (long long)ld_z, alpha, reinterpret_cast<__nv_bfloat16*>(s_scaled),
      reinterpret_cast<long long*>(keys), hdr.counter));
  return DELS_OK;
}

int dels_gather_scaled_rows_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* emb,
                                 int64_t ld_emb, const float* alpha, int n_pos, int B, int r, int V, void* s_scaled,
                                 int64_t* keys, void* ws, void* stream) {
  if (B < 0 || r <= 0 || V <= 0 || n_pos <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape");
  if (tokens == nullptr || emb == nullptr || s_scaled == nullptr) return fail(DELS_ERR_INVALID_ARG, "NULL argument");
  if (ld_emb < r) return fail(DELS_ERR_INVALID_ARG, "embedding leading dimension < r");
  unsigned* counter = ws != nullptr ? reinterpret_cast<unsigned*>(ws) : nullptr;
  int* status = ws != nullptr ? reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + 4) : nullptr;
  DeviceState* ds = nullptr;
  int rc;
  if ((rc = current_device_state(&ds)) != DELS_OK) return rc;
  if (B == 0) return DELS_OK;
  const int grid = cdiv((long long)B * r, 256) < 1024 ? cdiv((long long)B * r, 256) : 1024;
  DELS_CHECK_PDL("gather_scaled_kernel launch", launch_pdl(gather_scaled_kernel, dim3(grid), dim3(256), 0,
      reinterpret_cast<cudaStream_t>(stream), reinterpret_cast<const long long*>(tokens), tok_stride, token_keys,
      reinterpret_cast<const __nv_bfloat16*>(emb), ld_emb, alpha, n_pos, B, r, V,
      reinterpret_cast<__nv_bfloat16*>(s_scaled), reinterpret_cast<long long*>(keys), counter, status));
  return DELS_OK;
}

}  // extern "C"

// ======================================================================== allocation-free entry
//
// Some hosts cannot give this library device scratch memory: a service that binds the C
// ABI directly through an FFI layer (cgo, JNI, plain ctypes) has no device allocator of
// its own, and a serving engine that has already reserved nearly all of device memory
// for its KV-cache pool would see cudaMalloc fail, or pay for a device-wide
// synchronisation at the worst moment.  dels_draft_score_bf16_noalloc serves those
// callers: it runs exactly the dels_draft_score_bf16 kernels, with the scratch they
// need (packed keys, the scaled rank state, the split-K partial sums, the completion
// counter and the status word) placed in the fixed array below.  The array is part of
// the module image: it is reserved on every device on which the library's module is
// loaded, whether or not the entry point is ever called, and kept until the process
// exits.
//
// The array holds only the state of the call in flight: every call rewrites the keys,
// the rank state and the partials, and its rank-projection finalisation zeroes the
// completion counter before the scorer runs, so nothing carries over between calls
// except the status word (bytes [4, 8)), which a kernel that gives up on a bounded wait
// sets and which stays set until dels_noalloc_status clears it.  Calls that can overlap
// on the device (different streams, or different host threads without ordering) share
// the one array and race; serialise them.
namespace {

constexpr size_t kStaticScratchBytes = (size_t)DELS_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch in the current device's context.  The symbol's
// host-side name is a stand-in, not a device pointer, and must never reach a kernel.
// Looked up on every call (a host-side query, no stream work), so a context that was
// torn down and created again never sees a stale address.
int static_scratch_for_current_device(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
  if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255u) != 0)
    return fail(DELS_ERR_CUDA, "static scratch address is NULL or not 256-byte aligned");
  *out = p;
  return DELS_OK;
}

// One thread: copy the status word out, and clear it when asked.
__global__ void noalloc_status_kernel(int* word, int* out, int clear) {
  const int v = *reinterpret_cast<volatile int*>(word);
  if (out != nullptr) *out = v;
  if (clear) atomicExch(word, 0);
}

}  // namespace

extern "C" {

int dels_draft_score_bf16_noalloc(const void* h, int64_t ld_h, const void* W, int64_t ld_w, const void* w_rank,
                                  int64_t ld_wr, const void* Vr, int64_t ld_vr, const float* prior,
                                  const float* alpha, const float* beta, int n_pos, const int32_t* row_pos, int rows,
                                  const int32_t* rows_dev, int H, int r, int V, int64_t v_begin, int activation,
                                  int64_t* keys, int64_t* idx_out, float* score_out, void* stream) {
  if (rows < 0 || H <= 0 || r <= 0) return fail(DELS_ERR_INVALID_ARG, "bad shape rows=%d H=%d r=%d", rows, H, r);
  const size_t need = dels_score_workspace_bytes(rows, H, r);
  if (need > kStaticScratchBytes)
    return fail(DELS_ERR_WORKSPACE,
                "rows=%d, H=%d, r=%d need %zu bytes of scratch; the allocation-free entry point has %zu "
                "(use dels_draft_score_bf16 with a caller-provided workspace)",
                rows, H, r, need, kStaticScratchBytes);
  void* scratch = nullptr;
  int rc = static_scratch_for_current_device(&scratch);
  if (rc != DELS_OK) return rc;
  return dels_draft_score_bf16(h, ld_h, W, ld_w, w_rank, ld_wr, Vr, ld_vr, prior, alpha, beta, n_pos, row_pos, rows,
                               rows_dev, H, r, V, v_begin, activation, keys, idx_out, score_out, scratch,
                               kStaticScratchBytes, stream);
}

int dels_noalloc_status(int* status_out, int clear, void* stream) {
  if (status_out == nullptr && !clear) return fail(DELS_ERR_INVALID_ARG, "nothing to do: status_out NULL, clear 0");
  void* scratch = nullptr;
  int rc = static_scratch_for_current_device(&scratch);
  if (rc != DELS_OK) return rc;
  int* word = reinterpret_cast<int*>(reinterpret_cast<char*>(scratch) + 4);
  noalloc_status_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(word, status_out, clear ? 1 : 0);
  DELS_CHECK_LAUNCH("noalloc_status_kernel launch");
  return DELS_OK;
}

int dels_selftest_bounded_wait_noalloc(uint64_t* waited_ns, double limit_ms, void* stream) {
  void* scratch = nullptr;
  int rc = static_scratch_for_current_device(&scratch);
  if (rc != DELS_OK) return rc;
  return dels_selftest_bounded_wait(reinterpret_cast<int*>(reinterpret_cast<char*>(scratch) + 4), waited_ns,
                                    limit_ms, stream);
}

}  // extern "C"
