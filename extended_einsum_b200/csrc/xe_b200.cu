// C ABI of the sm_100a kernels (declared in include/xe_b200.h).  One
// translation unit so that the device status word is shared by all kernels.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/xe_b200.h"
#include "lse_gemm.cuh"
#include "cp_layer.cuh"
#include "cp_backward.cuh"
#include "tucker_layer.cuh"
#include "pointwise.cuh"

namespace {

thread_local std::string g_last_error;

xe_status fail(xe_status code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

xe_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(XE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return XE_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

int64_t grid_for(int64_t work, int64_t per_block, int64_t cap) {
  int64_t g = (work + per_block - 1) / per_block;
  return std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

constexpr size_t kAlign = 256;
inline size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// ------------------------------------------------------------------ GEMM
using xe::gemm::Params;

// Per-device "max dynamic shared memory" attribute, set once per kernel.
// `done_mask` must be distinct for every kernel (the callers pass a static of
// their own template instantiation).
template <typename K>
cudaError_t prepare_kernel(K kernel, int smem_bytes, std::atomic<uint32_t>& done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t bit = 1u << (dev & 31);
  if (done_mask.load() & bit) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e == cudaSuccess) done_mask.fetch_or(bit);
  return e;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::atomic<int> state{0};
  if (state.load() == 0) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && ptr) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
      state.store(1);
    } else {
      state.store(2);
    }
  }
  return fn;
}

// Tensor map of a (batch, rows, k) fp32 operand with k contiguous: boxes of
// 32 k x 128 rows, 128-byte swizzle (the layout load_staged_row reads).
bool encode_a_map(CUtensorMap* map, const float* base, int64_t batch, int64_t rows, int64_t k, int64_t s_row,
                  int64_t s_batch) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const int64_t sb = batch > 1 ? s_batch : rows * s_row;
  if (s_row <= 0 || sb <= 0 || (s_row * 4) % 16 != 0 || (sb * 4) % 16 != 0 || !aligned16(base)) return false;
  cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(s_row * 4), (cuuint64_t)(sb * 4)};
  cuuint32_t box[3] = {32, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map of a gather table viewed as `rows` rows of k fp32 (row stride s_row elements):
// boxes of one row x 32 k, 128-byte swizzle, for tile::gather4 loads of four rows each.
bool encode_gather_map(CUtensorMap* map, const float* base, int64_t rows, int64_t k, int64_t s_row) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode || !aligned16(base) || s_row <= 0 || (s_row * 4) % 16 != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(s_row * 4)};
  cuuint32_t box[2] = {32, 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map of a state table (folds, states, k) for whole-fold slabs: boxes of 32 k x all
// states (at most 256), 128-byte swizzle.
bool encode_slab_map(CUtensorMap* map, const float* base, int64_t folds, int64_t states, int64_t k, int64_t s_state,
                     int64_t s_fold) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode || !aligned16(base) || states > 256 || s_state <= 0 || s_fold <= 0 || (s_state * 4) % 16 != 0 ||
      (s_fold * 4) % 16 != 0)
    return false;
  cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)states, (cuuint64_t)folds};
  cuuint64_t strides[2] = {(cuuint64_t)(s_state * 4), (cuuint64_t)(s_fold * 4)};
  cuuint32_t box[3] = {32, (cuuint32_t)states, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map of the raw B operand (batch, k, n): MN-major (n contiguous) boxes
// of BN n x 32 k, K-major (k contiguous) boxes of 32 k x BN n; unswizzled.
bool encode_b_map(CUtensorMap* map, const float* base, int64_t batch, int64_t k, int64_t n, int64_t s_k, int64_t s_n,
                  int64_t s_batch, bool kmajor, int bn) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode || !aligned16(base)) return false;
  const int64_t s_outer = kmajor ? s_n : s_k;  // stride of the non-contiguous axis
  const int64_t rows = kmajor ? n : k;
  const int64_t sb = batch > 1 ? s_batch : rows * s_outer;
  if (s_outer <= 0 || sb <= 0 || (s_outer * 4) % 16 != 0 || (sb * 4) % 16 != 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)(kmajor ? k : n), (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(s_outer * 4), (cuuint64_t)(sb * 4)};
  cuuint32_t box[3] = {(cuuint32_t)(kmajor ? 32 : bn), (cuuint32_t)(kmajor ? bn : 32), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int AMODE, int ASRC, bool BK, int BSRC, int TJ>
xe_status launch_gemm_t(const Params& p, const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap& mb,
                        cudaStream_t stream) {
  using C = xe::gemm::Cfg<BN, ASRC, BSRC>;
  if constexpr (!C::kFits) {
    return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_gemm: staging configuration does not fit in shared memory");
  } else {
    auto kernel = xe::gemm::lse_gemm_kernel<BN, AMODE, ASRC, BK, BSRC, TJ>;
    static std::atomic<uint32_t> attribute_set{0};
    cudaError_t e = prepare_kernel(kernel, C::kSmemBytes, attribute_set);
    if (e != cudaSuccess) return fail(XE_ERR_CUDA, "xe_logspace_gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    const int grid = (int)std::min<int64_t>(p.num_tiles, current_device_sms());
    kernel<<<grid, C::kThreads, C::kSmemBytes, stream>>>(p, ma, ma2, mb);
    return check_launch("xe_logspace_gemm");
  }
}

template <int BN, int ASRC>
bool b_ring_fits() {
  using namespace xe::gemm;
  return Cfg<BN, ASRC, kBTma>::kFits;
}

template <int BN>
bool b_ring_fits_bn(int asrc) {
  using namespace xe::gemm;
  switch (asrc) {
    case kATma: return b_ring_fits<BN, kATma>();
    case kATma2: return b_ring_fits<BN, kATma2>();
    case kAGather: return b_ring_fits<BN, kAGather>();
    case kAGather2: return b_ring_fits<BN, kAGather2>();
    default: return b_ring_fits<BN, kALdg>();
  }
}

bool b_ring_fits(int bn, int asrc) {
  return bn == 128 ? b_ring_fits_bn<128>(asrc) : bn == 64 ? b_ring_fits_bn<64>(asrc) : b_ring_fits_bn<32>(asrc);
}

template <int BN, int AMODE, int ASRC>
xe_status launch_gemm_b(const Params& p, const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap& mb, bool bk,
                        int bsrc, cudaStream_t s) {
  using namespace xe::gemm;
  if (bk) {
    if (bsrc == kBTma) return launch_gemm_t<BN, AMODE, ASRC, true, kBTma, 0>(p, ma, ma2, mb, s);
    if (bsrc == kBLdgVec) return launch_gemm_t<BN, AMODE, ASRC, true, kBLdgVec, 0>(p, ma, ma2, mb, s);
    return launch_gemm_t<BN, AMODE, ASRC, true, kBLdg, 0>(p, ma, ma2, mb, s);
  }
  if (bsrc == kBTma) return launch_gemm_t<BN, AMODE, ASRC, false, kBTma, 0>(p, ma, ma2, mb, s);
  if (bsrc == kBLdgVec) return launch_gemm_t<BN, AMODE, ASRC, false, kBLdgVec, 0>(p, ma, ma2, mb, s);
  return launch_gemm_t<BN, AMODE, ASRC, false, kBLdg, 0>(p, ma, ma2, mb, s);
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

int pick_bn(int64_t n) {
  const int forced = env_int("XE_GEMM_BN", 0);
  if (forced == 32 || forced == 64 || forced == 128) return forced;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  return 128;
}

void set_tiling(Params& q, int bn) {
  q.tiles_m = (int)((q.M + xe::gemm::kBM - 1) / xe::gemm::kBM);
  q.tiles_n = (int)((q.N + bn - 1) / bn);
  q.num_tiles = q.tiles_m * q.tiles_n * q.batch;
  q.num_kb = (q.K + xe::gemm::kBK - 1) / xe::gemm::kBK;
}

// How one contraction runs: the tile width, where the A rows come from, and
// whether the A row shifts are computed in the kernel.
struct GemmPlan {
  int bn = 128;
  int asrc = xe::gemm::kALdg;
  int bsrc = xe::gemm::kBLdg;  // kBPlanes: B prepared by b_planes_kernel (Params::b_planes)
  bool inline_shift = false;
  CUtensorMap ma{};
  CUtensorMap ma2{};
  CUtensorMap mb{};
};

template <int BN, int ASRC>
int a_stages(int bsrc) {
  using namespace xe::gemm;
  return (bsrc == kBTma && Cfg<BN, ASRC, kBTma>::kFits) ? Cfg<BN, ASRC, kBTma>::kAStages : Cfg<BN, ASRC, kBLdg>::kAStages;
}

template <int BN>
int a_stages_bn(int asrc, int bsrc) {
  using namespace xe::gemm;
  switch (asrc) {
    case kATma: return a_stages<BN, kATma>(bsrc);
    case kATma2: return a_stages<BN, kATma2>(bsrc);
    case kAGather: return a_stages<BN, kAGather>(bsrc);
    case kAGather2: return a_stages<BN, kAGather2>(bsrc);
    default: return 0;
  }
}

int staged_k_capacity(int bn, int asrc, int bsrc) {
  using namespace xe::gemm;
  const int stages = bn == 128 ? a_stages_bn<128>(asrc, bsrc) : bn == 64 ? a_stages_bn<64>(asrc, bsrc) : a_stages_bn<32>(asrc, bsrc);
  return stages * kBK;
}

GemmPlan plan_gemm(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk, bool a_linear,
                   const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int64_t batch, int64_t m, int64_t n,
                   int64_t k, bool a_rows_gathered = false) {
  using namespace xe::gemm;
  GemmPlan g;
  g.bn = pick_bn(n);
  const bool no_tma = env_int("XE_GEMM_NO_TMA", 0) != 0;
  const bool a_tma = !no_tma && !a_rows_gathered && a_sk == 1 && (a_sm != 1 || m == 1) && encode_a_map(&g.ma, a, batch, m, k, a_sm, a_sb) &&
                     (a2 == nullptr || encode_a_map(&g.ma2, a2, batch, m, k, a_sm, a_sb));
  if (a_tma) g.asrc = a2 ? kATma2 : kATma;
  // B staging layout: K-major unless the N axis is the unit-stride one
  const bool bk = !(b_sn == 1) && b_sk == 1;
  const bool b_vec = aligned16(b) && b_sb % 4 == 0 &&
                     (bk ? (b_sk == 1 && k % 4 == 0 && b_sn % 4 == 0) : (b_sn == 1 && n % 4 == 0 && b_sk % 4 == 0));
  if (!no_tma && b_ring_fits(g.bn, g.asrc) && (bk ? b_sk == 1 : b_sn == 1) &&
      encode_b_map(&g.mb, b, batch, k, n, b_sk, b_sn, b_sb, bk, g.bn))
    g.bsrc = kBTma;
  else
    g.bsrc = b_vec ? kBLdgVec : kBLdg;
  const int inline_k = g.asrc == kALdg ? 128 : staged_k_capacity(g.bn, g.asrc, g.bsrc);
  g.inline_shift = !a_linear && k <= inline_k;
  return g;
}

// The gathered-row sources: K-major B staged by TMA or 16-byte loads only.
template <int BN, int ASRC>
xe_status launch_gemm_gather(const Params& q, const GemmPlan& g, cudaStream_t s) {
  using namespace xe::gemm;
  if (g.bsrc == kBTma) return launch_gemm_t<BN, kALog, ASRC, true, kBTma, 0>(q, g.ma, g.ma2, g.mb, s);
  return launch_gemm_t<BN, kALog, ASRC, true, kBLdgVec, 0>(q, g.ma, g.ma2, g.mb, s);
}

template <int ASRC>
xe_status launch_gemm_gather(const Params& q, const GemmPlan& g, cudaStream_t s) {
  return g.bn == 32 ? launch_gemm_gather<32, ASRC>(q, g, s)
                    : g.bn == 64 ? launch_gemm_gather<64, ASRC>(q, g, s) : launch_gemm_gather<128, ASRC>(q, g, s);
}

// Tensor map of an output (batch, m, n) with n contiguous: 32 x 32 blocks, 128-byte swizzle (TMA stores).
bool encode_c_map(CUtensorMap* map, float* base, int64_t batch, int64_t m, int64_t n, int64_t s_row, int64_t s_batch) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const int64_t sb = batch > 1 ? s_batch : m * s_row;
  if (s_row <= 0 || sb <= 0 || (s_row * 4) % 16 != 0 || (sb * 4) % 16 != 0 || !aligned16(base)) return false;
  cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)m, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(s_row * 4), (cuuint64_t)(sb * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int SRC>
xe_status launch_cp_layer_t(const xe::cp::Params& cp, const CUtensorMap& ma, const CUtensorMap& ma2,
                            const CUtensorMap& mb, const CUtensorMap& mc, cudaStream_t s) {
  constexpr int smem = xe::cp::Cfg<SRC>::kSmemBytes;
  auto kernel = xe::cp::cp_layer_kernel<SRC>;
  static std::atomic<uint32_t> attribute_set{0};
  cudaError_t e = prepare_kernel(kernel, smem, attribute_set);
  if (e != cudaSuccess) return fail(XE_ERR_CUDA, "xe_logspace_gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int grid = (int)std::min<int64_t>(cp.num_tiles, current_device_sms());
  kernel<<<grid, xe::cp::kThreads, smem, s>>>(cp, ma, ma2, mb, mc);
  return check_launch("xe_logspace_gemm");
}

xe_status launch_cp_layer(const xe::cp::Params& cp, int src, const CUtensorMap& ma, const CUtensorMap& ma2,
                          const CUtensorMap& mb, const CUtensorMap& mc, cudaStream_t s) {
  if (src == xe::cp::kSlab2) return launch_cp_layer_t<xe::cp::kSlab2>(cp, ma, ma2, mb, mc, s);
  if (src == xe::cp::kDense2) return launch_cp_layer_t<xe::cp::kDense2>(cp, ma, ma2, mb, mc, s);
  return launch_cp_layer_t<xe::cp::kDense>(cp, ma, ma2, mb, mc, s);
}

// The circuit's CP sum layer (K = N = 64, log A with its shifts computed in the kernel,
// linear K-major B staged by TMA, contiguous output, at least 4 tiles per fold) runs on
// its own kernel (cp_layer.cuh), which gives the same results as lse_gemm_kernel.
// XE_GEMM_NO_CP_LAYER=1 selects the general kernel.
xe_status try_cp_layer(const Params& q, const GemmPlan& g, bool a_linear, bool bk, cudaStream_t s, bool& launched) {
  using namespace xe::gemm;
  launched = false;
  if (a_linear || !bk || q.K != xe::cp::kK || q.N != xe::cp::kN || q.shift_b != nullptr || q.shift_a != nullptr ||
      q.raw_out || q.g_pixels != nullptr || (g.asrc != kATma && g.asrc != kATma2) || g.bsrc != kBTma || g.bn != 64 ||
      q.c_sn != 1 || q.tiles_m < 4 /* the weight split is per fold */ || env_int("XE_GEMM_NO_CP_LAYER", 0) != 0)
    return XE_OK;
  CUtensorMap mc{};
  if (!encode_c_map(&mc, q.c, q.batch, q.M, q.N, q.c_sm, q.c_sb)) return XE_OK;
  xe::cp::Params cp{};
  cp.folds = q.batch;
  cp.M = q.M;
  cp.tiles_m = q.tiles_m;
  cp.num_tiles = q.batch * q.tiles_m;
  cp.shift_min = q.shift_min;
  const int src = g.asrc == kATma2 ? xe::cp::kDense2 : xe::cp::kDense;
  launched = true;
  return launch_cp_layer(cp, src, g.ma, g.ma2, g.mb, mc, s);
}

// ------------------------------------------------------------------ prepared B
// The contraction with a prepared B operand (b_planes_kernel): 128-column tiles, B stages by bulk copy.
template <int ASRC>
constexpr bool planes_fit() {
  return xe::gemm::Cfg<128, ASRC, xe::gemm::kBPlanes>::kFits;
}

bool planes_fit_for(int asrc) {
  using namespace xe::gemm;
  return asrc == kATma ? planes_fit<kATma>() : asrc == kATma2 ? planes_fit<kATma2>() : asrc == kALdg ? planes_fit<kALdg>() : false;
}

xe_status launch_gemm_planes(const Params& q, const GemmPlan& g, bool a_linear, cudaStream_t s) {
  using namespace xe::gemm;
  if (g.bn != kPlaneN || !q.b_planes || !planes_fit_for(g.asrc))
    return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_gemm: prepared B needs 128-column tiles and a staged A");
  if (a_linear) {
    if (g.asrc == kATma) return launch_gemm_t<128, kALinear, kATma, true, kBPlanes, 0>(q, g.ma, g.ma2, g.mb, s);
    return launch_gemm_t<128, kALinear, kALdg, true, kBPlanes, 0>(q, g.ma, g.ma2, g.mb, s);
  }
  if (g.asrc == kATma) return launch_gemm_t<128, kALog, kATma, true, kBPlanes, 0>(q, g.ma, g.ma2, g.mb, s);
  if (g.asrc == kATma2) return launch_gemm_t<128, kALog, kATma2, true, kBPlanes, 0>(q, g.ma, g.ma2, g.mb, s);
  return launch_gemm_t<128, kALog, kALdg, true, kBPlanes, 0>(q, g.ma, g.ma2, g.mb, s);
}

// The prepared B: one kPlaneBlockBytes stage per (batch, 128-column tile, 32-k block), then the
// partial column extremes of the general preparation ([k slice][batch][tiles_n * 128] floats).
size_t planes_bytes(int64_t batch, int64_t n, int64_t k) {
  using namespace xe::gemm;
  const size_t tiles_n = (size_t)((n + kPlaneN - 1) / kPlaneN);
  const size_t stages = (size_t)batch * tiles_n * (size_t)((k + kBK - 1) / kBK) * (size_t)kPlaneBlockBytes;
  const size_t partials = (size_t)prep_ksplit((int)k) * (size_t)batch * tiles_n * kPlaneN * sizeof(float);
  return stages + round_up(partials);
}

size_t planes_stage_bytes(int64_t batch, int64_t n, int64_t k) {
  using namespace xe::gemm;
  return (size_t)batch * (size_t)((n + kPlaneN - 1) / kPlaneN) * (size_t)((k + kBK - 1) / kBK) * (size_t)kPlaneBlockBytes;
}

// How b_planes_kernel reads B: 1 = n contiguous, 2 = k contiguous (16-byte aligned rows both);
// 0 = not preparable.
int planes_layout(const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int64_t batch, int64_t n, int64_t k) {
  if (!aligned16(b) || (batch > 1 && b_sb % 4 != 0)) return 0;
  if (b_sn == 1 && n % 4 == 0 && b_sk % 4 == 0) return 1;
  if (b_sk == 1 && k % 4 == 0 && b_sn % 4 == 0) return 2;
  return 0;
}

// Whether xe_logspace_gemm prepares B (given the workspace): 128-column tiles (n > 64), at least
// kPlanesMinRowTiles row tiles of A and at least four k-blocks.  Preparing B costs one pass that
// reads B and writes twice its bytes; the kernel then runs about 13 % faster.  Measured on B200:
// 128 x 512^3 (4 row tiles) is 4 % slower with it, 8192^3 (64 row tiles) 7 % faster; the break-even
// is near 8 row tiles.  XE_GEMM_NO_PLANES=1 keeps the in-kernel B transform, XE_GEMM_PLANES=1
// prepares B whenever the shape allows.
constexpr int64_t kPlanesMinRowTiles = 8;
bool planes_pay(int64_t m, int64_t n, int64_t k) {
  if (env_int("XE_GEMM_NO_PLANES", 0) != 0 || pick_bn(n) != xe::gemm::kPlaneN || k <= 3 * xe::gemm::kBK) return false;
  const int64_t row_tiles = (m + xe::gemm::kBM - 1) / xe::gemm::kBM;
  return row_tiles >= (env_int("XE_GEMM_PLANES", 0) != 0 ? 2 : kPlanesMinRowTiles);
}

xe_status prepare_b(const char* who, const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, bool b_linear,
                    int64_t batch, int64_t n, int64_t k, bool maxmode, float* planes, float* shift_b, cudaStream_t s) {
  using namespace xe::gemm;
  const int lay = planes_layout(b, b_sb, b_sk, b_sn, batch, n, k);
  if (lay == 0)
    return fail(XE_ERR_NOT_SUPPORTED, "%s: B must have n or k contiguous, 16-byte aligned rows and a multiple of 4 "
                "along the contiguous axis", who);
  const int64_t tiles_n = (n + kPlaneN - 1) / kPlaneN;
  const int64_t grid = batch * tiles_n;
  if (grid > INT32_MAX) return fail(XE_ERR_NOT_SUPPORTED, "%s: too many B tiles", who);
  const int smin = maxmode ? 0 : 1;
  if (lay == 1 && k <= kStripeMaxK && grid * 4 <= INT32_MAX) {
    // n contiguous, short k: the whole column stripe of a CTA in shared memory, B read once
    const int smem = stripe_smem_bytes((int)k);
    // the attribute is set once per device, for the largest stripe
    static std::atomic<uint32_t> set_lin{0}, set_log{0};
    cudaError_t e = b_linear ? prepare_kernel(b_planes_stripe_kernel<false>, stripe_smem_bytes(kStripeMaxK), set_lin)
                             : prepare_kernel(b_planes_stripe_kernel<true>, stripe_smem_bytes(kStripeMaxK), set_log);
    if (e != cudaSuccess) return fail(XE_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", who, cudaGetErrorString(e));
    const unsigned g4 = (unsigned)(grid * 4);
    if (b_linear)
      b_planes_stripe_kernel<false><<<g4, 256, smem, s>>>(b, b_sb, b_sk, (int)n, (int)k, (int)tiles_n, smin, planes,
                                                          shift_b);
    else
      b_planes_stripe_kernel<true><<<g4, 256, smem, s>>>(b, b_sb, b_sk, (int)n, (int)k, (int)tiles_n, smin, planes,
                                                         shift_b);
    return check_launch(who);
  }
  // general preparation: partial column extremes over k slices, then the stages per k group
  float* partials = planes + planes_stage_bytes(batch, n, k) / sizeof(float);
  const int64_t ksplit = prep_ksplit((int)k);
  const int64_t groups = ((k + kBK - 1) / kBK + kPrepGroupKB - 1) / kPrepGroupKB;
  if (grid * ksplit > INT32_MAX || grid * groups > INT32_MAX) return fail(XE_ERR_NOT_SUPPORTED, "%s: too many B tiles", who);
  if (!b_linear) {
    const unsigned g1 = (unsigned)(grid * ksplit);
    if (lay == 1)
      b_col_extreme_kernel<false><<<g1, 256, 0, s>>>(b, b_sb, b_sk, b_sn, (int)n, (int)k, (int)tiles_n, (int)batch, smin,
                                                     partials);
    else
      b_col_extreme_kernel<true><<<g1, 256, 0, s>>>(b, b_sb, b_sk, b_sn, (int)n, (int)k, (int)tiles_n, (int)batch, smin,
                                                    partials);
  }
  const unsigned g = (unsigned)(grid * groups);
#define XE_PLANES(KM, LOG)                                                                                           \
  b_planes_kernel<KM, LOG><<<g, 256, 0, s>>>(b, b_sb, b_sk, b_sn, (int)n, (int)k, (int)tiles_n, (int)batch, smin, \
                                             partials, planes, shift_b)
  if (lay == 1) {
    if (b_linear) XE_PLANES(false, false);
    else XE_PLANES(false, true);
  } else {
    if (b_linear) XE_PLANES(true, false);
    else XE_PLANES(true, true);
  }
#undef XE_PLANES
  return check_launch(who);
}

xe_status launch_gemm(const Params& p, const GemmPlan& g, bool a_linear, bool bk, cudaStream_t s) {
  using namespace xe::gemm;
  Params q = p;
  set_tiling(q, g.bn);
  if (g.bsrc == kBPlanes) return launch_gemm_planes(q, g, a_linear, s);
  if (q.batch > 0 && q.M > 0) {
    bool launched = false;
    const xe_status st = try_cp_layer(q, g, a_linear, bk, s, launched);
    if (launched || st != XE_OK) return st;
  }
  if (a_gathered(g.asrc)) {
    if (a_linear || !bk || g.bsrc == kBLdg)
      return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_gemm_gather: staged gather needs a log table and K-major B");
    return g.asrc == kAGather ? launch_gemm_gather<kAGather>(q, g, s) : launch_gemm_gather<kAGather2>(q, g, s);
  }
#define XE_LAUNCH_BN(BN)                                                                                           \
  do {                                                                                                             \
    if (a_linear) {                                                                                                \
      if (g.asrc == kATma) return launch_gemm_b<BN, kALinear, kATma>(q, g.ma, g.ma2, g.mb, bk, g.bsrc, s);         \
      return launch_gemm_b<BN, kALinear, kALdg>(q, g.ma, g.ma2, g.mb, bk, g.bsrc, s);                              \
    }                                                                                                              \
    if (g.asrc == kATma) return launch_gemm_b<BN, kALog, kATma>(q, g.ma, g.ma2, g.mb, bk, g.bsrc, s);              \
    if (g.asrc == kATma2) return launch_gemm_b<BN, kALog, kATma2>(q, g.ma, g.ma2, g.mb, bk, g.bsrc, s);            \
    return launch_gemm_b<BN, kALog, kALdg>(q, g.ma, g.ma2, g.mb, bk, g.bsrc, s);                                   \
  } while (0)
  switch (g.bn) {
    case 32: XE_LAUNCH_BN(32);
    case 64: XE_LAUNCH_BN(64);
    default: XE_LAUNCH_BN(128);
  }
#undef XE_LAUNCH_BN
}

xe_status shift_impl(const float* x, const float* x2, int64_t sb, int64_t sr, int64_t sk, int64_t batch, int64_t rows,
                     int64_t k, bool maxmode, float* out, cudaStream_t stream) {
  if (batch == 0 || rows == 0) return XE_OK;
  const bool al = aligned16(x) && (x2 == nullptr || aligned16(x2));
  if (sr == 1 && sk != 1) {
    const bool vec = al && rows % 4 == 0 && sk % 4 == 0 && sb % 4 == 0;
    dim3 block(32, 8), grid((unsigned)((rows + 127) / 128), (unsigned)batch);
    if (maxmode) {
      if (vec) xe::shift_rows_colwise<true, true><<<grid, block, 0, stream>>>(x, x2, sb, sk, rows, k, out);
      else xe::shift_rows_colwise<true, false><<<grid, block, 0, stream>>>(x, x2, sb, sk, rows, k, out);
    } else {
      if (vec) xe::shift_rows_colwise<false, true><<<grid, block, 0, stream>>>(x, x2, sb, sk, rows, k, out);
      else xe::shift_rows_colwise<false, false><<<grid, block, 0, stream>>>(x, x2, sb, sk, rows, k, out);
    }
  } else {
    const bool vec = al && sk == 1 && k % 4 == 0 && sr % 4 == 0 && sb % 4 == 0;
    const int64_t warps = batch * rows;
    const int64_t blocks = (warps + 7) / 8;
    if (maxmode) {
      if (vec) xe::shift_rows_warp<true, true><<<(unsigned)blocks, 256, 0, stream>>>(x, x2, sb, sr, sk, batch, rows, k, out);
      else xe::shift_rows_warp<true, false><<<(unsigned)blocks, 256, 0, stream>>>(x, x2, sb, sr, sk, batch, rows, k, out);
    } else {
      if (vec) xe::shift_rows_warp<false, true><<<(unsigned)blocks, 256, 0, stream>>>(x, x2, sb, sr, sk, batch, rows, k, out);
      else xe::shift_rows_warp<false, false><<<(unsigned)blocks, 256, 0, stream>>>(x, x2, sb, sr, sk, batch, rows, k, out);
    }
  }
  return check_launch("xe_logspace_shift");
}

bool make_nd(const int64_t* shape, const int64_t* as, const int64_t* bs, int ndim, xe::NdShape& sh, int64_t& total,
             bool& contig) {
  sh = xe::NdShape{};
  sh.ndim = ndim;
  total = 1;
  contig = true;
  int64_t expect = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    if (shape[d] < 0) return false;
    sh.shape[d] = shape[d];
    sh.as[d] = as[d];
    sh.bs[d] = bs[d];
    if (shape[d] != 1 && (as[d] != expect || bs[d] != expect)) contig = false;
    expect *= shape[d];
    total *= shape[d];
  }
  if (ndim == 0) {
    sh.ndim = 1;
    sh.shape[0] = 1;
    sh.as[0] = sh.bs[0] = 0;
  }
  return true;
}

}  // namespace

// The log-space Tucker layer 'bfi,bfj,foij->bfo' (defined after the C entry points).
static xe_status xe_tucker_impl(const float* l, int64_t l_sb, int64_t l_sf, const float* r, int64_t r_sb,
                                int64_t r_sf, const float* w, float* y, int64_t y_sb, int64_t y_sf, int64_t batch,
                                int64_t folds, int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode,
                                cudaStream_t stream);

namespace xe {
// The bounded-wait test kernel (xe_wait_probe): warp 0 waits on a barrier expecting one
// arrival; with `complete` set, warp 1 arrives after a bounded delay, otherwise nothing
// arrives and the wait runs out after g_wait_timeout_ns.
__global__ void wait_probe_kernel(int complete) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    mbar_wait(&bar, 0, kSiteWaitProbe, &abort_flag);
  } else if (threadIdx.x == 32 && complete) {
    const long long t0 = clock64();
    while (clock64() - t0 < 20000) {
    }
    mbar_arrive(&bar);
  }
}
}  // namespace xe

extern "C" {

int xe_version(void) { return 100; }

xe_status xe_set_wait_timeout_ns(uint64_t ns) {
  const uint64_t value = ns == 0 ? xe::kWaitTimeoutNs : ns;
  if (value < 1000ull || value > 60000000000ull)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_set_wait_timeout_ns: %llu ns is outside [1 us, 60 s]",
                (unsigned long long)ns);
  const cudaError_t e = cudaMemcpyToSymbol(xe::g_wait_timeout_ns, &value, sizeof(value));
  if (e != cudaSuccess) return fail(XE_ERR_CUDA, "xe_set_wait_timeout_ns: %s", cudaGetErrorString(e));
  return XE_OK;
}

xe_status xe_wait_probe(int complete, void* stream) {
  xe::wait_probe_kernel<<<1, 64, 0, as_stream(stream)>>>(complete);
  return check_launch("xe_wait_probe");
}

const char* xe_last_error_string(void) { return g_last_error.c_str(); }

int xe_device_status(int clear) {
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fail(XE_ERR_CUDA, "xe_device_status: %s", cudaGetErrorString(e));
    return XE_ERR_CUDA << 16;
  }
  e = cudaMemcpyFromSymbol(&v, xe::g_device_status, sizeof(int));
  if (e != cudaSuccess) {
    fail(XE_ERR_CUDA, "xe_device_status: %s", cudaGetErrorString(e));
    return XE_ERR_CUDA << 16;
  }
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(xe::g_device_status, &zero, sizeof(int));
  }
  return v;
}

#ifdef XE_TRACE_TILES
// Trace builds only: copies (and clears) the CP-layer kernel's per-tile event times of CTA 0.
int xe_profile_trace(long long* out, int n) {
  const int count = n < xe::kTraceTiles * xe::kTraceEvents ? n : xe::kTraceTiles * xe::kTraceEvents;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(out, xe::g_trace, count * sizeof(long long)) != cudaSuccess) return -1;
  static long long zero[xe::kTraceTiles * xe::kTraceEvents] = {};
  cudaMemcpyToSymbol(xe::g_trace, zero, sizeof(zero));
  return count;
}
#endif

#ifdef XE_PROFILE
// Profiling builds only: copies (and optionally clears) the per-site wait-cycle counters.
int xe_profile_wait_cycles(unsigned long long* out, int n, int clear) {
  const int count = n < xe::kNumSites ? n : xe::kNumSites;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(out, xe::g_wait_cycles, count * sizeof(unsigned long long)) != cudaSuccess) return -1;
  if (n >= 2 * xe::kNumSites &&
      cudaMemcpyFromSymbol(out + xe::kNumSites, xe::g_segment_cycles, xe::kNumSites * sizeof(unsigned long long)) !=
          cudaSuccess)
    return -1;
  if (clear) {
    unsigned long long zero[xe::kNumSites] = {};
    cudaMemcpyToSymbol(xe::g_wait_cycles, zero, sizeof(zero));
    cudaMemcpyToSymbol(xe::g_segment_cycles, zero, sizeof(zero));
  }
  return count;
}
#endif

size_t xe_logspace_gemm_workspace_size(int64_t batch, int64_t m, int64_t n, int64_t k, int32_t a_linear,
                                       int32_t b_linear) {
  (void)k;
  size_t bytes = 0;
  if (!a_linear) bytes += round_up((size_t)batch * (size_t)m * sizeof(float));
  if (!b_linear) bytes += round_up((size_t)batch * (size_t)n * sizeof(float));
  return bytes;
}

xe_status xe_logspace_shift(const float* x, const float* x2, int64_t sb, int64_t sr, int64_t sk, int64_t batch,
                            int64_t rows, int64_t k, int32_t shift_mode, float* out, void* stream) {
  if (!x || !out) return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_shift: null pointer");
  if (batch < 0 || rows < 0 || k <= 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_shift: the reduced axis must be non-empty (k=%lld)", (long long)k);
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_shift: unknown shift mode %d", shift_mode);
  return shift_impl(x, x2, sb, sr, sk, batch, rows, k, shift_mode == XE_SHIFT_MAX, out, as_stream(stream));
}

}  // extern "C"

namespace {

// A rows gathered by uint8 pixel values (categorical input units, see Params::g_pixels).
struct GatherA {
  const uint8_t* pixels;
  const int32_t* var;
  int64_t stride;
  int states;
  int64_t pair;  // > 0: the row of fold + pair is added (Params::g_pair)
};

xe_status gemm_launch(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk, bool a_linear,
                      const float* shift_a, const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                      const float* shift_b, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t batch, int64_t m,
                      int64_t n, int64_t k, bool shift_min, const GemmPlan& g, cudaStream_t s,
                      bool raw_out = false, const GatherA* gather = nullptr, const float* b_planes = nullptr,
                      const int64_t* shift_strides = nullptr) {
  Params p{};
  p.b_planes = b_planes;
  p.a = a;
  p.a2 = a2;
  p.a_sb = a_sb;
  p.a_sm = a_sm;
  p.a_sk = a_sk;
  p.b = b;
  p.b_sb = b_sb;
  p.b_sk = b_sk;
  p.b_sn = b_sn;
  p.c = c;
  p.c_sb = c_sb;
  p.c_sm = c_sm;
  p.c_sn = c_sn;
  p.shift_a = shift_a;
  p.shift_b = shift_b;
  p.sa_sb = m;
  p.sa_sm = 1;
  p.sb_sb = n;
  p.sb_sn = 1;
  if (shift_strides) {
    p.sa_sb = shift_strides[0];
    p.sa_sm = shift_strides[1];
    p.sb_sb = shift_strides[2];
    p.sb_sn = shift_strides[3];
  }
  p.batch = (int)batch;
  p.M = (int)m;
  p.N = (int)n;
  p.K = (int)k;
  p.c_vec = (c_sn == 1 && n % 4 == 0 && c_sm % 4 == 0 && c_sb % 4 == 0 && aligned16(c)) ? 1 : 0;
  p.a_vec = (a_sk == 1 && k % 4 == 0 && a_sm % 4 == 0 && a_sb % 4 == 0 && aligned16(a) &&
             (a2 == nullptr || aligned16(a2))) ? 1 : 0;
  p.shift_min = shift_min ? 1 : 0;
  p.raw_out = raw_out ? 1 : 0;
  if (gather) {
    p.g_pixels = gather->pixels;
    p.g_var = gather->var;
    p.g_stride = gather->stride;
    p.g_states = gather->states;
    p.g_pair = gather->pair;
    p.a_vec = (k % 4 == 0 && a_sm % 4 == 0 && a_sb % 4 == 0 && aligned16(a)) ? 1 : 0;
  }
  const bool bk = !(b_sn == 1) && b_sk == 1;
  return launch_gemm(p, g, a_linear, bk, s);
}

xe_status gemm_check(const char* who, const float* a, const float* b, const float* c, int64_t batch, int64_t m,
                     int64_t n, int64_t k) {
  if (!a || !b || !c) return fail(XE_ERR_INVALID_ARGUMENT, "%s: null operand pointer", who);
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(XE_ERR_INVALID_ARGUMENT, "%s: negative extent", who);
  if (k == 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: the contracted extent is empty (reduction over size 0)", who);
  if (batch > INT32_MAX || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return fail(XE_ERR_NOT_SUPPORTED, "%s: extents above 2^31-1 are not supported", who);
  return XE_OK;
}

}  // namespace

extern "C" {

xe_status xe_logspace_gemm(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk, int32_t a_linear,
                           const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int32_t b_linear, float* c,
                           int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t batch, int64_t m, int64_t n, int64_t k,
                           int32_t shift_mode, void* workspace, size_t workspace_bytes, void* stream) {
  xe_status st = gemm_check("xe_logspace_gemm", a, b, c, batch, m, n, k);
  if (st != XE_OK) return st;
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm: unknown shift mode %d", shift_mode);
  if (a2 && a_linear)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm: a fused addend requires a log-domain A operand");
  if (batch == 0 || m == 0 || n == 0) return XE_OK;
  const size_t need = xe_logspace_gemm_workspace_size(batch, m, n, k, a_linear, b_linear);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm: workspace of %zu bytes required, %zu given", need,
                workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm: workspace must be 256-byte aligned");

  cudaStream_t s = as_stream(stream);
  const bool maxmode = shift_mode == XE_SHIFT_MAX;
  float* ws = static_cast<float*>(workspace);
  float* shift_a = nullptr;
  float* shift_b = nullptr;
  GemmPlan plan = plan_gemm(a, a2, a_sb, a_sm, a_sk, a_linear != 0, b, b_sb, b_sk, b_sn, batch, m, n, k);
  // B prepared once (b_planes_kernel) when the workspace also holds it, after the shift vectors
  if (planes_pay(m, n, k) && planes_layout(b, b_sb, b_sk, b_sn, batch, n, k) != 0 && planes_fit_for(plan.asrc) &&
      !plan.inline_shift && workspace_bytes >= need + planes_bytes(batch, n, k)) {
    float* planes = reinterpret_cast<float*>(static_cast<char*>(workspace) + need);
    if (!a_linear) {
      shift_a = ws;
      st = shift_impl(a, a2, a_sb, a_sm, a_sk, batch, m, k, maxmode, shift_a, s);
      if (st != XE_OK) return st;
      ws = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + round_up((size_t)batch * m * sizeof(float)));
    }
    shift_b = b_linear ? nullptr : ws;
    st = prepare_b("xe_logspace_gemm", b, b_sb, b_sk, b_sn, b_linear != 0, batch, n, k, maxmode, planes, shift_b, s);
    if (st != XE_OK) return st;
    plan.bn = xe::gemm::kPlaneN;
    plan.bsrc = xe::gemm::kBPlanes;
    return gemm_launch(a, a2, a_sb, a_sm, a_sk, a_linear != 0, shift_a, b, b_sb, b_sk, b_sn, shift_b, c, c_sb, c_sm,
                       c_sn, batch, m, n, k, !maxmode, plan, s, false, nullptr, planes);
  }
  if (!a_linear) {
    // small K: the kernel computes the row shifts itself (shift_a stays null)
    if (!plan.inline_shift) {
      shift_a = ws;
      st = shift_impl(a, a2, a_sb, a_sm, a_sk, batch, m, k, maxmode, shift_a, s);
      if (st != XE_OK) return st;
    }
    ws = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + round_up((size_t)batch * m * sizeof(float)));
  }
  if (!b_linear) {
    shift_b = ws;
    st = shift_impl(b, nullptr, b_sb, b_sn, b_sk, batch, n, k, maxmode, shift_b, s);
    if (st != XE_OK) return st;
  }
  return gemm_launch(a, a2, a_sb, a_sm, a_sk, a_linear != 0, shift_a, b, b_sb, b_sk, b_sn, shift_b, c, c_sb, c_sm,
                     c_sn, batch, m, n, k, !maxmode, plan, s);
}

// ------------------------------------------------------------------------
// Allocation-free variant: the shift vectors live in this static array.
static __device__ __align__(256) float g_noalloc_scratch[XE_NOALLOC_SCRATCH_BYTES / sizeof(float)];

}  // extern "C"

namespace {

std::mutex g_noalloc_mutex;
void* g_noalloc_scratch_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device, resolved once per
// device.  In host code the array's name is only a stand-in for the symbol.
xe_status noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(XE_ERR_CUDA, "xe_logspace_gemm_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_gemm_noalloc: device index %d above 63", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(XE_ERR_CUDA, "xe_logspace_gemm_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_scratch_ptr[dev] = ptr;
  }
  *out = g_noalloc_scratch_ptr[dev];
  return XE_OK;
}

}  // namespace

extern "C" {

xe_status xe_logspace_gemm_noalloc(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                   int32_t a_linear, const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                                   int32_t b_linear, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t batch,
                                   int64_t m, int64_t n, int64_t k, int32_t shift_mode, void* stream) {
  if (batch < 0 || m < 0 || n < 0 || k < 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_noalloc: negative extent");
  const size_t need = xe_logspace_gemm_workspace_size(batch, m, n, k, a_linear, b_linear);
  if (need > XE_NOALLOC_SCRATCH_BYTES)
    return fail(XE_ERR_INVALID_ARGUMENT,
                "xe_logspace_gemm_noalloc: the shift vectors need %zu bytes, above the %u-byte static scratch "
                "(batch*(m+n) too large); use xe_logspace_gemm with a workspace",
                need, (unsigned)XE_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  xe_status st = noalloc_scratch(&scratch);
  if (st != XE_OK) return st;
  return xe_logspace_gemm(a, a2, a_sb, a_sm, a_sk, a_linear, b, b_sb, b_sk, b_sn, b_linear, c, c_sb, c_sm, c_sn, batch,
                          m, n, k, shift_mode, scratch, XE_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"

namespace {

// The sum layer over gathered table rows; pair > 0 adds the row of fold f + pair.
xe_status gather_gemm(const char* who, const float* table, int64_t t_sf, int64_t t_ss, int64_t states,
                      const uint8_t* pixels, int64_t pixel_stride, const int32_t* var_of_fold, int64_t pair,
                      const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int32_t b_linear, float* c,
                      int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t folds, int64_t batch, int64_t n, int64_t k,
                      int32_t shift_mode, void* workspace, size_t workspace_bytes, void* stream) {
  xe_status st = gemm_check(who, table, b, c, folds, batch, n, k);
  if (st != XE_OK) return st;
  if (!pixels) return fail(XE_ERR_INVALID_ARGUMENT, "%s: null pixels", who);
  if (states <= 0 || states > 256)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: uint8 pixels address 1 to 256 states (got %lld)", who, (long long)states);
  if (pixel_stride <= 0) return fail(XE_ERR_INVALID_ARGUMENT, "%s: pixel_stride must be positive", who);
  if (pair < 0) return fail(XE_ERR_INVALID_ARGUMENT, "%s: negative fold offset %lld", who, (long long)pair);
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: unknown shift mode %d", who, shift_mode);
  if (k > 128)
    return fail(XE_ERR_NOT_SUPPORTED, "%s: at most 128 units per input row (got %lld)", who, (long long)k);
  if (folds == 0 || batch == 0 || n == 0) return XE_OK;
  const size_t need = xe_logspace_gemm_workspace_size(folds, batch, n, k, 1, b_linear);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes required, %zu given", who, need, workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: workspace must be 256-byte aligned", who);
  cudaStream_t s = as_stream(stream);
  float* shift_b = nullptr;
  if (!b_linear) {
    shift_b = static_cast<float*>(workspace);
    st = shift_impl(b, nullptr, b_sb, b_sn, b_sk, folds, n, k, shift_mode == XE_SHIFT_MAX, shift_b, s);
    if (st != XE_OK) return st;
  }
  // the second CP sum layer of a circuit over a state table: the CP-layer kernel with the
  // two folds' table slabs in shared memory (same results as the general kernel below)
  if (pair > 0 && k == xe::cp::kK && n == xe::cp::kN && b_linear && b_sk == 1 && b_sn != 1 && c_sn == 1 &&
      states <= 256 && (batch + xe::gemm::kBM - 1) / xe::gemm::kBM >= 4 && env_int("XE_GEMM_NO_CP_LAYER", 0) == 0) {
    CUtensorMap slab{}, mw{}, mc{};
    if (encode_slab_map(&slab, table, folds + pair, states, k, t_ss, t_sf) &&
        encode_b_map(&mw, b, folds, k, n, b_sk, b_sn, b_sb, true, xe::cp::kN) &&
        encode_c_map(&mc, c, folds, batch, n, c_sm, c_sb)) {
      xe::cp::Params cp{};
      cp.folds = (int)folds;
      cp.M = (int)batch;
      cp.tiles_m = (int)((batch + xe::gemm::kBM - 1) / xe::gemm::kBM);
      cp.num_tiles = cp.folds * cp.tiles_m;
      cp.shift_min = shift_mode == XE_SHIFT_MIN ? 1 : 0;
      cp.pixels = pixels;
      cp.var = var_of_fold;
      cp.pixel_stride = pixel_stride;
      cp.states = (int)states;
      cp.pair = (int)pair;
      return launch_cp_layer(cp, xe::cp::kSlab2, slab, slab, mw, mc, s);
    }
  }
  // the A rows are gathered per thread (global loads), their shifts computed in the kernel
  GemmPlan plan = plan_gemm(table, nullptr, t_sf, t_ss, 1, false, b, b_sb, b_sk, b_sn, folds, batch, n, k, true);
  plan.inline_shift = true;
  const bool bk = !(b_sn == 1) && b_sk == 1;
  // rows staged by TMA gather loads when the table is (folds * states) rows of 16-byte aligned stride
  const int64_t table_rows = (folds + pair) * states;
  if (env_int("XE_GEMM_NO_TMA", 0) == 0 && t_sf == states * t_ss && bk && table_rows <= INT32_MAX &&
      encode_gather_map(&plan.ma, table, table_rows, k, t_ss)) {
    using namespace xe::gemm;
    const int asrc = pair > 0 ? kAGather2 : kAGather;
    int bsrc = plan.bsrc;
    if (bsrc == kBTma && !b_ring_fits(plan.bn, asrc)) bsrc = kBLdgVec;
    const bool b_vec = aligned16(b) && b_sb % 4 == 0 && k % 4 == 0 && b_sn % 4 == 0;
    if (bsrc != kBTma && b_vec) bsrc = kBLdgVec;
    // the in-kernel row shift needs every k-block of a tile staged at once
    if ((bsrc == kBTma || bsrc == kBLdgVec) && k <= staged_k_capacity(plan.bn, asrc, bsrc)) {
      plan.asrc = asrc;
      plan.bsrc = bsrc == kBTma ? kBTma : kBLdgVec;
    }
  }
  const GatherA gather{pixels, var_of_fold, pixel_stride, (int)states, pair};
  return gemm_launch(table, nullptr, t_sf, t_ss, 1, false, nullptr, b, b_sb, b_sk, b_sn, shift_b, c, c_sb, c_sm, c_sn,
                     folds, batch, n, k, shift_mode == XE_SHIFT_MIN, plan, s, false, &gather);
}

}  // namespace

extern "C" {

xe_status xe_logspace_gemm_gather(const float* table, int64_t t_sf, int64_t t_ss, int64_t states, const uint8_t* pixels,
                                  int64_t pixel_stride, const int32_t* var_of_fold, const float* b, int64_t b_sb,
                                  int64_t b_sk, int64_t b_sn, int32_t b_linear, float* c, int64_t c_sb, int64_t c_sm,
                                  int64_t c_sn, int64_t folds, int64_t batch, int64_t n, int64_t k, int32_t shift_mode,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  return gather_gemm("xe_logspace_gemm_gather", table, t_sf, t_ss, states, pixels, pixel_stride, var_of_fold, 0, b,
                     b_sb, b_sk, b_sn, b_linear, c, c_sb, c_sm, c_sn, folds, batch, n, k, shift_mode, workspace,
                     workspace_bytes, stream);
}

xe_status xe_logspace_gemm_gather_pair(const float* table, int64_t t_sf, int64_t t_ss, int64_t states,
                                       const uint8_t* pixels, int64_t pixel_stride, const int32_t* var_of_fold,
                                       int64_t fold_offset, const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                                       int32_t b_linear, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                       int64_t folds, int64_t batch, int64_t n, int64_t k, int32_t shift_mode,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  if (fold_offset <= 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_gather_pair: fold_offset must be positive (got %lld)",
                (long long)fold_offset);
  return gather_gemm("xe_logspace_gemm_gather_pair", table, t_sf, t_ss, states, pixels, pixel_stride, var_of_fold,
                     fold_offset, b, b_sb, b_sk, b_sn, b_linear, c, c_sb, c_sm, c_sn, folds, batch, n, k, shift_mode,
                     workspace, workspace_bytes, stream);
}

xe_status xe_logspace_gemm_shifted(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                   const float* shift_a, const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                                   const float* shift_b, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                   int64_t batch, int64_t m, int64_t n, int64_t k, void* stream) {
  xe_status st = gemm_check("xe_logspace_gemm_shifted", a, b, c, batch, m, n, k);
  if (st != XE_OK) return st;
  if (a2 && !shift_a)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_shifted: a fused addend requires a log-domain A operand");
  if (batch == 0 || m == 0 || n == 0) return XE_OK;
  GemmPlan plan = plan_gemm(a, a2, a_sb, a_sm, a_sk, shift_a == nullptr, b, b_sb, b_sk, b_sn, batch, m, n, k);
  plan.inline_shift = false;
  return gemm_launch(a, a2, a_sb, a_sm, a_sk, shift_a == nullptr, shift_a, b, b_sb, b_sk, b_sn, shift_b, c, c_sb, c_sm,
                     c_sn, batch, m, n, k, false, plan, as_stream(stream));
}

xe_status xe_logspace_gemm_shifted_strided(const float* a, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                           const float* shift_a, int64_t sa_sb, int64_t sa_sm, const float* b,
                                           int64_t b_sb, int64_t b_sk, int64_t b_sn, const float* shift_b,
                                           int64_t sb_sb, int64_t sb_sn, float* c, int64_t c_sb, int64_t c_sm,
                                           int64_t c_sn, int64_t batch, int64_t m, int64_t n, int64_t k, void* stream) {
  xe_status st = gemm_check("xe_logspace_gemm_shifted_strided", a, b, c, batch, m, n, k);
  if (st != XE_OK) return st;
  if (!shift_a || !shift_b)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_shifted_strided: both operands are log-domain: shifts required");
  if (sa_sb < 0 || sa_sm < 0 || sb_sb < 0 || sb_sn < 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_shifted_strided: negative shift stride");
  if (batch == 0 || m == 0 || n == 0) return XE_OK;
  GemmPlan plan = plan_gemm(a, nullptr, a_sb, a_sm, a_sk, false, b, b_sb, b_sk, b_sn, batch, m, n, k);
  plan.inline_shift = false;
  const int64_t strides[4] = {sa_sb, sa_sm, sb_sb, sb_sn};
  return gemm_launch(a, nullptr, a_sb, a_sm, a_sk, false, shift_a, b, b_sb, b_sk, b_sn, shift_b, c, c_sb, c_sm, c_sn,
                     batch, m, n, k, false, plan, as_stream(stream), false, nullptr, nullptr, strides);
}

size_t xe_logspace_b_prepared_size(int64_t batch, int64_t n, int64_t k) {
  if (batch <= 0 || n <= 0 || k <= 0) return 0;
  return planes_bytes(batch, n, k);
}

size_t xe_logspace_gemm_workspace_size_prepared(int64_t batch, int64_t m, int64_t n, int64_t k, int32_t a_linear,
                                                int32_t b_linear) {
  const size_t base = xe_logspace_gemm_workspace_size(batch, m, n, k, a_linear, b_linear);
  if (batch <= 0 || m <= 0 || n <= 0 || k <= 0 || !planes_pay(m, n, k)) return base;
  return base + planes_bytes(batch, n, k);
}

xe_status xe_logspace_b_prepare(const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int32_t b_linear,
                                int64_t batch, int64_t n, int64_t k, int32_t shift_mode, float* prepared,
                                size_t prepared_bytes, float* shift_b, void* stream) {
  if (!b || !prepared) return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_b_prepare: null pointer");
  if (!b_linear && !shift_b)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_b_prepare: a log-domain B needs a shift_b output");
  if (batch < 0 || n < 0 || k <= 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_b_prepare: the contracted extent must be non-empty (k=%lld)",
                (long long)k);
  if (batch > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_b_prepare: extents above 2^31-1 are not supported");
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_b_prepare: unknown shift mode %d", shift_mode);
  if (batch == 0 || n == 0) return XE_OK;
  if (prepared_bytes < planes_bytes(batch, n, k))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_b_prepare: %zu bytes needed for the prepared B, %zu given",
                planes_bytes(batch, n, k), prepared_bytes);
  if (!aligned16(prepared)) return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_b_prepare: prepared must be 16-byte aligned");
  return prepare_b("xe_logspace_b_prepare", b, b_sb, b_sk, b_sn, b_linear != 0, batch, n, k,
                   shift_mode == XE_SHIFT_MAX, prepared, b_linear ? nullptr : shift_b, as_stream(stream));
}

xe_status xe_logspace_gemm_prepared(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                    const float* shift_a, const float* prepared, const float* shift_b, float* c,
                                    int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t batch, int64_t m, int64_t n,
                                    int64_t k, void* stream) {
  xe_status st = gemm_check("xe_logspace_gemm_prepared", a, prepared, c, batch, m, n, k);
  if (st != XE_OK) return st;
  if (a2 && !shift_a)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_prepared: a fused addend requires a log-domain A operand");
  if (!aligned16(prepared))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_gemm_prepared: prepared must be 16-byte aligned");
  if (batch == 0 || m == 0 || n == 0) return XE_OK;
  // A staged by TMA where its layout allows (the B arguments only steer the plan's A part)
  GemmPlan plan = plan_gemm(a, a2, a_sb, a_sm, a_sk, shift_a == nullptr, prepared, 0, 1, k, batch, m, n, k);
  plan.inline_shift = false;
  if (!planes_fit_for(plan.asrc)) plan.asrc = xe::gemm::kALdg;
  plan.bn = xe::gemm::kPlaneN;
  plan.bsrc = xe::gemm::kBPlanes;
  return gemm_launch(a, a2, a_sb, a_sm, a_sk, shift_a == nullptr, shift_a, prepared, 0, 1, k, shift_b, c, c_sb, c_sm,
                     c_sn, batch, m, n, k, false, plan, as_stream(stream), false, nullptr, prepared);
}

xe_status xe_softmax(const float* x, float* y, int64_t outer, int64_t axis_len, int64_t inner, int32_t log_output,
                     void* stream) {
  if (!x || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_softmax: null pointer");
  if (outer < 0 || axis_len < 0 || inner < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_softmax: negative extent");
  if (outer == 0 || axis_len == 0 || inner == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  const int lo = log_output ? 1 : 0;
  if (inner > 1) {
    if (inner % 4 == 0 && inner <= 256 && 256 % inner == 0 && axis_len * inner <= xe::kSlabMaxFloats &&
        aligned16(x) && aligned16(y) && outer <= INT32_MAX && env_int("XE_SOFTMAX_NO_SLAB", 0) == 0) {
      // one outer slice per CTA, staged in shared memory
      const int smem = (int)((axis_len * inner + 256 + 2 * inner) * sizeof(float));
      static std::atomic<uint32_t> attribute_set{0};
      cudaError_t e = prepare_kernel(xe::softmax_slab, (xe::kSlabMaxFloats + 256 + 2 * 256) * (int)sizeof(float),
                                     attribute_set);
      if (e != cudaSuccess) return fail(XE_ERR_CUDA, "xe_softmax: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      xe::softmax_slab<<<(unsigned)outer, 256, smem, s>>>(x, y, axis_len, (int)inner, lo);
      return check_launch("xe_softmax");
    }
    const int64_t fibres = outer * inner;
    xe::softmax_strided<<<(unsigned)((fibres + 255) / 256), 256, 0, s>>>(x, y, outer, axis_len, inner, lo);
    return check_launch("xe_softmax");
  }
  const bool vec = aligned16(x) && aligned16(y) && axis_len % 4 == 0;
  const int64_t rows = outer, len = axis_len;
  if (vec && len <= 64) {
    // short rows: a group of lanes per row, several rows per warp
#define XE_SOFTMAX_GROUP(G) \
  xe::softmax_rows_group<G><<<(unsigned)((rows * G + 255) / 256), 256, 0, s>>>(x, y, rows, len, lo)
    if (len <= 4) XE_SOFTMAX_GROUP(1);
    else if (len <= 8) XE_SOFTMAX_GROUP(2);
    else if (len <= 16) XE_SOFTMAX_GROUP(4);
    else if (len <= 32) XE_SOFTMAX_GROUP(8);
    else XE_SOFTMAX_GROUP(16);
#undef XE_SOFTMAX_GROUP
    return check_launch("xe_softmax");
  }
#define XE_SOFTMAX_WARP(Q)                                                                                   \
  do {                                                                                                       \
    const unsigned blocks = (unsigned)((rows + 7) / 8);                                                      \
    if (vec) xe::softmax_rows_reg<32, Q, true><<<blocks, 256, 0, s>>>(x, y, rows, len, lo);                   \
    else xe::softmax_rows_reg<32, Q, false><<<blocks, 256, 0, s>>>(x, y, rows, len, lo);                      \
  } while (0)
#define XE_SOFTMAX_BLOCK(T, Q)                                                                               \
  do {                                                                                                       \
    if (vec) xe::softmax_rows_reg<T, Q, true><<<(unsigned)rows, T, 0, s>>>(x, y, rows, len, lo);              \
    else xe::softmax_rows_reg<T, Q, false><<<(unsigned)rows, T, 0, s>>>(x, y, rows, len, lo);                 \
  } while (0)
  if (len <= 128) XE_SOFTMAX_WARP(1);
  else if (len <= 512) XE_SOFTMAX_WARP(4);
  else if (len <= 1024) XE_SOFTMAX_WARP(8);
  else if (len <= 4096) XE_SOFTMAX_BLOCK(256, 4);
  else if (len <= 16384) XE_SOFTMAX_BLOCK(1024, 4);
  else if (len <= 32768 && vec && env_int("XE_SOFTMAX_NO_PREFETCH", 0) == 0) {
    // one row in registers while the next one streams into shared memory
    const int smem = (int)(len * 4);
    static std::atomic<uint32_t> attribute_set{0};
    cudaError_t e = prepare_kernel(xe::softmax_rows_prefetch<8>, 32768 * 4, attribute_set);  // the largest row
    if (e != cudaSuccess) return fail(XE_ERR_CUDA, "xe_softmax: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    const int grid = (int)std::min<int64_t>(rows, current_device_sms());
    xe::softmax_rows_prefetch<8><<<grid, 1024, smem, s>>>(x, y, rows, len, lo);
  } else if (len <= 32768) XE_SOFTMAX_BLOCK(1024, 8);
  else if (len <= 65536) XE_SOFTMAX_BLOCK(1024, 16);
  else xe::softmax_rows_stream<<<(unsigned)rows, 1024, 0, s>>>(x, y, len, lo);
#undef XE_SOFTMAX_WARP
#undef XE_SOFTMAX_BLOCK
  return check_launch("xe_softmax");
}

xe_status xe_log_add(const float* a, const int64_t* a_strides, const float* b, const int64_t* b_strides, float* y,
                     const int64_t* shape, int32_t ndim, int32_t negate_b, void* stream) {
  if (!a || !b || !y || !shape || !a_strides || !b_strides) return fail(XE_ERR_INVALID_ARGUMENT, "xe_log_add: null pointer");
  if (ndim < 0 || ndim > 6) return fail(XE_ERR_NOT_SUPPORTED, "xe_log_add: rank %d above 6 is not supported", ndim);
  xe::NdShape sh{};
  int64_t total = 0;
  bool contig = false;
  if (!make_nd(shape, a_strides, b_strides, ndim, sh, total, contig)) return fail(XE_ERR_INVALID_ARGUMENT, "xe_log_add: negative extent");
  if (total == 0) return XE_OK;
  const float sign = negate_b ? -1.0f : 1.0f;
  cudaStream_t s = as_stream(stream);
  const int cap = current_device_sms() * 8;
  if (contig && total % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(y)) {
    const int64_t n4 = total / 4;
    xe::log_add_contig4<<<(unsigned)grid_for(n4, 256, cap), 256, 0, s>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(y), n4, sign);
  } else {
    xe::log_add_nd<<<(unsigned)grid_for(total, 256, cap), 256, 0, s>>>(a, b, y, sh, total, sign);
  }
  return check_launch("xe_log_add");
}

xe_status xe_categorical_gather(const float* table, const uint8_t* pixels, int64_t pixel_stride,
                                const int32_t* var_of_fold, float* y, int64_t folds, int64_t states, int64_t units,
                                int64_t batch, void* stream) {
  if (!table || !pixels || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_categorical_gather: null pointer");
  if (folds < 0 || states <= 0 || units < 0 || batch < 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_categorical_gather: invalid extents");
  if (states > 256) return fail(XE_ERR_INVALID_ARGUMENT, "xe_categorical_gather: uint8 pixels address at most 256 states");
  if (folds == 0 || units == 0 || batch == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  const int cap = current_device_sms() * 8;
  if (units % 4 == 0 && aligned16(table) && aligned16(y)) {
    const int64_t total = folds * batch * (units / 4);
    xe::categorical_gather4<<<(unsigned)grid_for(total, 256, cap), 256, 0, s>>>(table, pixels, pixel_stride, var_of_fold,
                                                                                y, folds, states, units, batch);
  } else {
    const int64_t total = folds * batch * units;
    xe::categorical_gather1<<<(unsigned)grid_for(total, 256, cap), 256, 0, s>>>(table, pixels, pixel_stride, var_of_fold,
                                                                                y, folds, states, units, batch);
  }
  return check_launch("xe_categorical_gather");
}

xe_status xe_categorical_scatter_add(const float* grad, const uint8_t* pixels, int64_t pixel_stride,
                                     const int32_t* var_of_fold, float* table_grad, int64_t folds, int64_t states,
                                     int64_t units, int64_t batch, int64_t fold_offset, void* stream) {
  if (!grad || !pixels || !table_grad) return fail(XE_ERR_INVALID_ARGUMENT, "xe_categorical_scatter_add: null pointer");
  if (folds < 0 || states <= 0 || units < 0 || batch < 0 || fold_offset < 0 || pixel_stride <= 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_categorical_scatter_add: invalid extents");
  if (states > 256)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_categorical_scatter_add: uint8 pixels address at most 256 states");
  if (folds == 0 || units == 0 || batch == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  const int64_t smem = states * units * (int64_t)sizeof(float);
  if (smem <= 96 * 1024) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
      const cudaError_t e =
          cudaFuncSetAttribute(xe::categorical_scatter_smem, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      if (e != cudaSuccess)
        return fail(XE_ERR_CUDA, "xe_categorical_scatter_add: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr_set[dev] = true;
    }
    // at least two CTAs per SM: the batch is split into chunks when there are few folds
    const int64_t target = 2 * (int64_t)current_device_sms();
    const int64_t chunks = std::max<int64_t>(1, std::min<int64_t>(batch, (target + folds - 1) / folds));
    const int64_t b_chunk = (batch + chunks - 1) / chunks;
    dim3 grid((unsigned)folds, (unsigned)((batch + b_chunk - 1) / b_chunk));
    xe::categorical_scatter_smem<<<grid, 256, (size_t)smem, s>>>(grad, pixels, pixel_stride, var_of_fold, table_grad,
                                                                  states, units, batch, fold_offset, b_chunk);
  } else {
    const int64_t total = folds * batch * units;
    xe::categorical_scatter_global<<<(unsigned)grid_for(total, 256, current_device_sms() * 8), 256, 0, s>>>(
        grad, pixels, pixel_stride, var_of_fold, table_grad, folds, states, units, batch, fold_offset);
  }
  return check_launch("xe_categorical_scatter_add");
}

xe_status xe_logspace_reduce(const float* x, int64_t sb, int64_t sr, int64_t sk, int64_t batch, int64_t rows, int64_t k,
                             int32_t shift_mode, float* y, void* stream) {
  if (!x || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_reduce: null pointer");
  if (batch < 0 || rows < 0 || k <= 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_reduce: the reduced axes must be non-empty (k=%lld)", (long long)k);
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_reduce: unknown shift mode %d", shift_mode);
  if (batch == 0 || rows == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  const bool mx = shift_mode == XE_SHIFT_MAX;
  if (sr == 1 && sk != 1) {
    dim3 block(32, 8), grid((unsigned)((rows + 31) / 32), (unsigned)batch);
    if (mx) xe::lse_rows_colwise<true><<<grid, block, 0, s>>>(x, sb, sk, rows, k, y);
    else xe::lse_rows_colwise<false><<<grid, block, 0, s>>>(x, sb, sk, rows, k, y);
  } else {
    const bool vec = aligned16(x) && sk == 1 && k % 4 == 0 && sr % 4 == 0 && sb % 4 == 0;
    const unsigned blocks = (unsigned)((batch * rows + 7) / 8);
    if (mx) {
      if (vec) xe::lse_rows_warp<true, true><<<blocks, 256, 0, s>>>(x, sb, sr, sk, batch, rows, k, y);
      else xe::lse_rows_warp<true, false><<<blocks, 256, 0, s>>>(x, sb, sr, sk, batch, rows, k, y);
    } else {
      if (vec) xe::lse_rows_warp<false, true><<<blocks, 256, 0, s>>>(x, sb, sr, sk, batch, rows, k, y);
      else xe::lse_rows_warp<false, false><<<blocks, 256, 0, s>>>(x, sb, sr, sk, batch, rows, k, y);
    }
  }
  return check_launch("xe_logspace_reduce");
}

xe_status xe_log_add_exp(const float* a, const int64_t* a_strides, int64_t a_numel, const float* b,
                         const int64_t* b_strides, int64_t b_numel, float* y, const int64_t* shape, int32_t ndim,
                         int32_t subtract, int32_t shift_mode, float* scratch, void* stream) {
  if (!a || !b || !y || !shape || !a_strides || !b_strides || !scratch)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_log_add_exp: null pointer");
  if (ndim < 0 || ndim > 6) return fail(XE_ERR_NOT_SUPPORTED, "xe_log_add_exp: rank %d above 6 is not supported", ndim);
  if (a_numel <= 0 || b_numel <= 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_log_add_exp: empty operand");
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_log_add_exp: unknown shift mode %d", shift_mode);
  xe::NdShape sh{};
  int64_t total = 0;
  bool contig = false;
  if (!make_nd(shape, a_strides, b_strides, ndim, sh, total, contig))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_log_add_exp: negative extent");
  if (total == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  if (shift_mode == XE_SHIFT_MAX) xe::global_extreme2<true><<<1, 1024, 0, s>>>(a, a_numel, b, b_numel, scratch);
  else xe::global_extreme2<false><<<1, 1024, 0, s>>>(a, a_numel, b, b_numel, scratch);
  const int cap = current_device_sms() * 8;
  xe::log_add_exp_nd<<<(unsigned)grid_for(total, 256, cap), 256, 0, s>>>(a, b, y, sh, total, scratch, subtract ? 1 : 0);
  return check_launch("xe_log_add_exp");
}

xe_status xe_unary(const float* x, float* y, int64_t n, int32_t op, void* stream) {
  if (!x || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_unary: null pointer");
  if (op != 0 && op != 1) return fail(XE_ERR_INVALID_ARGUMENT, "xe_unary: unknown op %d", op);
  if (n < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_unary: negative extent");
  if (n == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  const int cap = current_device_sms() * 8;
  if (n % 4 == 0 && aligned16(x) && aligned16(y)) {
    const int64_t n4 = n / 4;
    const unsigned g = (unsigned)grid_for(n4, 256, cap);
    if (op == 0) xe::unary_map4<0><<<g, 256, 0, s>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n4);
    else xe::unary_map4<1><<<g, 256, 0, s>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n4);
  } else {
    const unsigned g = (unsigned)grid_for(n, 256, cap);
    if (op == 0) xe::unary_map<0><<<g, 256, 0, s>>>(x, y, n);
    else xe::unary_map<1><<<g, 256, 0, s>>>(x, y, n);
  }
  return check_launch("xe_unary");
}

xe_status xe_logspace_tucker(const float* l, const float* r, const float* w, float* y, int64_t batch, int64_t folds,
                             int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode, void* stream) {
  return xe_tucker_impl(l, folds * i_dim, i_dim, r, folds * j_dim, j_dim, w, y, folds * o_dim, o_dim, batch, folds, i_dim,
                        j_dim, o_dim, shift_mode, as_stream(stream));
}

xe_status xe_logspace_tucker_strided(const float* l, int64_t l_sb, int64_t l_sf, const float* r, int64_t r_sb,
                                     int64_t r_sf, const float* w, float* y, int64_t y_sb, int64_t y_sf, int64_t batch,
                                     int64_t folds, int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode,
                                     void* stream) {
  return xe_tucker_impl(l, l_sb, l_sf, r, r_sb, r_sf, w, y, y_sb, y_sf, batch, folds, i_dim, j_dim, o_dim, shift_mode,
                        as_stream(stream));
}

}  // extern "C"

template <int TJ>
xe_status launch_tucker(const Params& p, cudaStream_t s) {
  using namespace xe::gemm;
  const int bn = pick_bn(p.N);
  Params q = p;
  set_tiling(q, bn);
  const CUtensorMap none{};
  CUtensorMap mb{};
  const bool b_tma = env_int("XE_GEMM_NO_TMA", 0) == 0 &&
                     encode_b_map(&mb, p.b, p.batch, p.K, p.N, p.b_sk, p.b_sn, p.b_sb, true, bn);
#define XE_TUCKER_BN(BN)                                                                   \
  return b_tma ? launch_gemm_t<BN, kATucker, kALdg, true, kBTma, TJ>(q, none, none, mb, s) \
               : launch_gemm_t<BN, kATucker, kALdg, true, kBLdgVec, TJ>(q, none, none, mb, s)
  switch (bn) {
    case 32: XE_TUCKER_BN(32);
    case 64: XE_TUCKER_BN(64);
    default: XE_TUCKER_BN(128);
  }
#undef XE_TUCKER_BN
}

static xe_status xe_tucker_impl(const float* l, int64_t l_sb, int64_t l_sf, const float* r, int64_t r_sb,
                                int64_t r_sf, const float* w, float* y, int64_t y_sb, int64_t y_sf, int64_t batch,
                                int64_t folds, int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode,
                                cudaStream_t stream) {
  if (!l || !r || !w || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_tucker: null pointer");
  if (batch < 0 || folds < 0 || i_dim <= 0 || j_dim <= 0 || o_dim < 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_tucker: invalid extents");
  // l and r rows are loaded as 16-byte vectors or through tensor maps: each starts on 16 bytes
  for (const int64_t stride : {l_sb, l_sf, r_sb, r_sf})
    if (stride < 0 || stride % 4 != 0)
      return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_tucker: l and r row strides must be non-negative multiples of 4");
  if (y_sb < 0 || y_sf < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_tucker: negative output strides");
  // output rows of 16-byte multiples: the Tucker kernel's tensor-map stores and vector stores
  const bool y_rows16 = y_sb % 4 == 0 && y_sf % 4 == 0;
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_tucker: unknown shift mode %d", shift_mode);
  if ((j_dim != 32 && j_dim != 64) || i_dim % 8 != 0)
    return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_tucker: J must be 32 or 64 and I a multiple of 8 (got I=%lld, J=%lld)",
                (long long)i_dim, (long long)j_dim);
  if (batch > INT32_MAX || folds > INT32_MAX || i_dim * j_dim > INT32_MAX || o_dim > INT32_MAX)
    return fail(XE_ERR_NOT_SUPPORTED, "xe_logspace_tucker: extents above 2^31-1 are not supported");
  if (!aligned16(l) || !aligned16(r) || !aligned16(w))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_logspace_tucker: operands must be 16-byte aligned");
  if (batch == 0 || folds == 0 || o_dim == 0) return XE_OK;
  // I = J = O = 32: the two-stage kernel (tucker_layer.cuh); XE_GEMM_NO_CP_LAYER=1 selects the general one
  if (i_dim == xe::tk::kDim && j_dim == xe::tk::kDim && o_dim == xe::tk::kDim && y_rows16 && aligned16(y) &&
      env_int("XE_GEMM_NO_CP_LAYER", 0) == 0) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    CUtensorMap ml{}, mr{}, mw{}, my{};
    bool maps = encode != nullptr;
    auto rows_map = [&](CUtensorMap* map, const float* base, int box_rows, int64_t s_b, int64_t s_f) {
      // (batch, folds, 32) with 32 contiguous units per row: boxes of 32 x 1 fold x box_rows rows,
      // 128-byte swizzle
      cuuint64_t dims[3] = {32, (cuuint64_t)folds, (cuuint64_t)batch};
      cuuint64_t strides[2] = {(cuuint64_t)(s_f * 4), (cuuint64_t)(s_b * 4)};
      cuuint32_t box[3] = {32, 1, (cuuint32_t)box_rows};
      cuuint32_t estr[3] = {1, 1, 1};
      return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    if (maps)
      maps = rows_map(&ml, l, xe::gemm::kBM, l_sb, l_sf) && rows_map(&mr, r, xe::gemm::kBM, r_sb, r_sf) &&
             rows_map(&my, y, 32, y_sb, y_sf);
    if (maps) {
      // w (folds, 32 o, 32 i, 32 j): per fold 1024 (o,i) rows of 32 j; chunks of 64 rows
      cuuint64_t dims[3] = {32, 1024, (cuuint64_t)folds};
      cuuint64_t strides[2] = {32 * 4, 1024 * 32 * 4};
      cuuint32_t box[3] = {32, xe::tk::kChunkN, 1};
      cuuint32_t estr[3] = {1, 1, 1};
      maps = encode(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (maps) {
      xe::tk::Params tp{};
      tp.rows = (int)batch;
      tp.folds = (int)folds;
      tp.tiles_m = (int)((batch + xe::gemm::kBM - 1) / xe::gemm::kBM);
      tp.num_tiles = tp.folds * tp.tiles_m;
      tp.shift_min = shift_mode == XE_SHIFT_MIN;
      static std::atomic<uint32_t> attribute_set{0};
      cudaError_t e = prepare_kernel(xe::tk::tucker_layer_kernel, xe::tk::Cfg::kSmemBytes, attribute_set);
      if (e != cudaSuccess)
        return fail(XE_ERR_CUDA, "xe_logspace_tucker: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      const int grid = (int)std::min<int64_t>(tp.num_tiles, current_device_sms());
      xe::tk::tucker_layer_kernel<<<grid, xe::tk::kThreads, xe::tk::Cfg::kSmemBytes, stream>>>(tp, ml, mr, mw, my);
      return check_launch("xe_logspace_tucker");
    }
  }
  Params p{};
  // the weights are the linear, K-major B operand of a batched contraction over folds
  p.b = w;
  p.b_sb = o_dim * i_dim * j_dim;
  p.b_sk = 1;
  p.b_sn = i_dim * j_dim;
  p.c = y;
  p.c_sb = y_sf;
  p.c_sm = y_sb;
  p.c_sn = 1;
  p.batch = (int)folds;
  p.M = (int)batch;
  p.N = (int)o_dim;
  p.K = (int)(i_dim * j_dim);
  p.c_vec = (o_dim % 4 == 0 && y_rows16 && aligned16(y)) ? 1 : 0;
  p.tl = l;
  p.tr = r;
  p.t_folds = (int)folds;
  p.t_i = (int)i_dim;
  p.t_l_sb = l_sb;
  p.t_l_sf = l_sf;
  p.t_r_sb = r_sb;
  p.t_r_sf = r_sf;
  p.shift_min = shift_mode == XE_SHIFT_MIN;
  return j_dim == 32 ? launch_tucker<32>(p, stream) : launch_tucker<64>(p, stream);
}

// ------------------------------------------------------------------------
// Scaled stability modes.

namespace {

template <int OP>
void launch_elementwise(const float* a, const float* b, const float* c, float* y, const xe::NdShape3& sh, int64_t total,
                        bool contig, cudaStream_t s) {
  const int cap = current_device_sms() * 8;
  if (contig && total % 4 == 0 && aligned16(a) && (!b || aligned16(b)) && (!c || aligned16(c)) && aligned16(y)) {
    const int64_t n4 = total / 4;
    xe::elementwise_contig4<OP><<<(unsigned)grid_for(n4, 256, cap), 256, 0, s>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), reinterpret_cast<const float4*>(c),
        reinterpret_cast<float4*>(y), n4);
  } else if (sh.ndim >= 1 && sh.shape[sh.ndim - 1] >= 32) {
    const int64_t n = sh.shape[sh.ndim - 1];
    const int64_t rows = total / n;
    xe::elementwise_rows<OP><<<(unsigned)grid_for(rows, 8, (int64_t)current_device_sms() * 16), 256, 0, s>>>(
        a, b, c, y, sh, rows, n);
  } else {
    xe::elementwise_nd<OP><<<(unsigned)grid_for(total, 256, cap), 256, 0, s>>>(a, b, c, y, sh, total);
  }
}

template <int KIND>
void launch_fiber(const float* x, const xe::RowIndexer& ri, int64_t rows, int64_t n, int64_t sn, float* normalized,
                  float* log_scale, cudaStream_t s) {
  const int64_t blocks = grid_for(rows, 8, (int64_t)current_device_sms() * 16);
  xe::fiber_rows<KIND><<<(unsigned)blocks, 256, 0, s>>>(x, ri, rows, n, sn, normalized, log_scale);
}

template <int KIND>
void launch_reduce(const float* x, int64_t sb, int64_t sr, int64_t sk, int64_t batch, int64_t rows, int64_t k, float* y,
                   cudaStream_t s) {
  // contiguous outputs, a strided k at least 64 long, one block per batch entry (at least 64 of
  // them): columns across threads (coalesced loads)
  if (sr == 1 && rows <= 256 && sk >= rows && k >= 64 && batch >= 64 && batch <= INT32_MAX) {
    xe::reduce_cols<KIND><<<(unsigned)batch, 1024, 0, s>>>(x, sb, sk, rows, k, y);
    return;
  }
  const int64_t blocks = grid_for(batch * rows, 8, (int64_t)current_device_sms() * 16);
  xe::reduce_rows<KIND><<<(unsigned)blocks, 256, 0, s>>>(x, sb, sr, sk, batch, rows, k, y);
}

}  // namespace

extern "C" {

xe_status xe_scaled_gemm(const float* a, int64_t a_sb, int64_t a_sm, int64_t a_sk, const float* b, int64_t b_sb,
                         int64_t b_sk, int64_t b_sn, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t batch,
                         int64_t m, int64_t n, int64_t k, void* stream) {
  xe_status st = gemm_check("xe_scaled_gemm", a, b, c, batch, m, n, k);
  if (st != XE_OK) return st;
  if (batch == 0 || m == 0 || n == 0) return XE_OK;
  const GemmPlan plan = plan_gemm(a, nullptr, a_sb, a_sm, a_sk, true, b, b_sb, b_sk, b_sn, batch, m, n, k);
  return gemm_launch(a, nullptr, a_sb, a_sm, a_sk, true, nullptr, b, b_sb, b_sk, b_sn, nullptr, c, c_sb, c_sm, c_sn,
                     batch, m, n, k, false, plan, as_stream(stream), true);
}

xe_status xe_fiber_normalize(const float* x, const int64_t* shape, const int64_t* strides, int32_t ndim, int32_t kind,
                             float* normalized, float* log_scale, void* stream) {
  if (!x || !normalized || !log_scale || (ndim > 0 && (!shape || !strides)))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_fiber_normalize: null pointer");
  if (ndim < 0 || ndim > 7) return fail(XE_ERR_NOT_SUPPORTED, "xe_fiber_normalize: rank %d above 7 is not supported", ndim);
  if (kind < XE_FIBER_SUM || kind > XE_FIBER_LSE) return fail(XE_ERR_INVALID_ARGUMENT, "xe_fiber_normalize: unknown kind %d", kind);
  xe::RowIndexer ri{};
  int64_t rows = 1, n = 1, sn = 0;
  if (ndim > 0) {
    n = shape[ndim - 1];
    sn = strides[ndim - 1];
    ri.ndim = ndim - 1;
    for (int d = 0; d < ndim - 1; ++d) {
      if (shape[d] < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_fiber_normalize: negative extent");
      ri.shape[d] = shape[d];
      ri.stride[d] = strides[d];
      rows *= shape[d];
    }
    if (n < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_fiber_normalize: negative extent");
  }
  if (ri.ndim == 0) {
    ri.ndim = 1;
    ri.shape[0] = 1;
    ri.stride[0] = 0;
  }
  if (n == 0 && kind != XE_FIBER_SUM && kind != XE_FIBER_LSE && rows > 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_fiber_normalize: max/min of an empty fibre");
  if (rows == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  switch (kind) {
    case XE_FIBER_SUM: launch_fiber<xe::kFiberSum>(x, ri, rows, n, sn, normalized, log_scale, s); break;
    case XE_FIBER_MAX: launch_fiber<xe::kFiberMax>(x, ri, rows, n, sn, normalized, log_scale, s); break;
    case XE_FIBER_MIN: launch_fiber<xe::kFiberMin>(x, ri, rows, n, sn, normalized, log_scale, s); break;
    case XE_FIBER_EXP: launch_fiber<xe::kFiberExp>(x, ri, rows, n, sn, normalized, log_scale, s); break;
    default: launch_fiber<xe::kFiberLse>(x, ri, rows, n, sn, normalized, log_scale, s); break;
  }
  return check_launch("xe_fiber_normalize");
}

xe_status xe_reduce(const float* x, int64_t sb, int64_t sr, int64_t sk, int64_t batch, int64_t rows, int64_t k,
                    int32_t kind, float* y, void* stream) {
  if (!x || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_reduce: null pointer");
  if (batch < 0 || rows < 0 || k < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_reduce: negative extent");
  if (kind != XE_FIBER_SUM && kind != XE_FIBER_MAX && kind != XE_FIBER_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_reduce: unknown kind %d", kind);
  if (k == 0 && kind != XE_FIBER_SUM && batch * rows > 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_reduce: max/min over an empty axis");
  if (batch == 0 || rows == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  if (kind == XE_FIBER_SUM) launch_reduce<xe::kFiberSum>(x, sb, sr, sk, batch, rows, k, y, s);
  else if (kind == XE_FIBER_MAX) launch_reduce<xe::kFiberMax>(x, sb, sr, sk, batch, rows, k, y, s);
  else launch_reduce<xe::kFiberMin>(x, sb, sr, sk, batch, rows, k, y, s);
  return check_launch("xe_reduce");
}

xe_status xe_elementwise(int32_t op, const float* a, const int64_t* a_strides, const float* b, const int64_t* b_strides,
                         const float* c, const int64_t* c_strides, float* y, const int64_t* shape, int32_t ndim,
                         void* stream) {
  if (op < XE_OP_ADD || op > XE_OP_RESCALE) return fail(XE_ERR_INVALID_ARGUMENT, "xe_elementwise: unknown op %d", op);
  const bool needs_c = op == XE_OP_RESCALE;
  if (!a || !b || !y || (needs_c && !c) || (ndim > 0 && (!shape || !a_strides || !b_strides || (needs_c && !c_strides))))
    return fail(XE_ERR_INVALID_ARGUMENT, "xe_elementwise: null pointer");
  if (ndim < 0 || ndim > 6) return fail(XE_ERR_NOT_SUPPORTED, "xe_elementwise: rank %d above 6 is not supported", ndim);
  if (!needs_c) c = nullptr;
  xe::NdShape3 sh{};
  sh.ndim = ndim;
  int64_t total = 1, expect = 1;
  bool contig = true;
  for (int d = ndim - 1; d >= 0; --d) {
    if (shape[d] < 0) return fail(XE_ERR_INVALID_ARGUMENT, "xe_elementwise: negative extent");
    sh.shape[d] = shape[d];
    sh.as[d] = a_strides[d];
    sh.bs[d] = b_strides[d];
    sh.cs[d] = c ? c_strides[d] : 0;
    if (shape[d] != 1 && (sh.as[d] != expect || sh.bs[d] != expect || (c && sh.cs[d] != expect))) contig = false;
    expect *= shape[d];
    total *= shape[d];
  }
  if (ndim == 0) {
    sh.ndim = 1;
    sh.shape[0] = 1;
  }
  if (total == 0) return XE_OK;
  cudaStream_t s = as_stream(stream);
  switch (op) {
    case XE_OP_ADD: launch_elementwise<xe::kOpAdd>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_SUB: launch_elementwise<xe::kOpSub>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_MUL: launch_elementwise<xe::kOpMul>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_DIV: launch_elementwise<xe::kOpDiv>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_MAX: launch_elementwise<xe::kOpMax>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_MIN: launch_elementwise<xe::kOpMin>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_MUL_EXP: launch_elementwise<xe::kOpMulExp>(a, b, c, y, sh, total, contig, s); break;
    case XE_OP_LOG_ADD: launch_elementwise<xe::kOpLogAdd>(a, b, c, y, sh, total, contig, s); break;
    default: launch_elementwise<xe::kOpRescale>(a, b, c, y, sh, total, contig, s); break;
  }
  return check_launch("xe_elementwise");
}

}  // extern "C"

// ------------------------------------------------------------------ CP layer backward
namespace {

// Tensor map of a contiguous (folds, m, 64) operand: boxes of 32 columns x 32 rows, 128-byte swizzle.
bool encode_rows_map(CUtensorMap* map, const float* base, int64_t folds, int64_t m) {
  return encode_c_map(map, const_cast<float*>(base), folds, m, 64, 64, m * 64);
}

struct CpbGeometry {
  int64_t tiles_m = 0, num_tiles = 0;
  int grid = 0, pieces = 0;
};

// The tiles, the grid (one CTA per SM at most) and the workspace slots per fold: the most CTAs
// whose tile ranges meet one fold.
CpbGeometry cpb_geometry(int64_t folds, int64_t m) {
  using xe::cpb::cta_of_tile;
  CpbGeometry g;
  g.tiles_m = (m + xe::cpb::kRows - 1) / xe::cpb::kRows;
  g.num_tiles = folds * g.tiles_m;
  if (g.num_tiles == 0) return g;
  g.grid = (int)std::min<int64_t>(g.num_tiles, current_device_sms());
  g.pieces = 1;
  for (int64_t f = 0; f < folds; ++f) {
    const int c0 = cta_of_tile(f * g.tiles_m, g.num_tiles, g.grid);
    const int c1 = cta_of_tile(f * g.tiles_m + g.tiles_m - 1, g.num_tiles, g.grid);
    g.pieces = std::max(g.pieces, c1 - c0 + 1);
  }
  return g;
}

size_t cpb_workspace_bytes(const CpbGeometry& g, int64_t folds) {
  return g.num_tiles == 0 ? 0 : round_up((size_t)folds * (size_t)g.pieces * 2 * 4096 * sizeof(float));
}

template <int SRC>
xe_status launch_cpb_t(const char* who, const xe::cpb::Params& q, const CUtensorMap& mx1, const CUtensorMap& mx2,
                       const CUtensorMap& my, const CUtensorMap& mg, int grid, cudaStream_t s) {
  auto kernel = xe::cpb::cpb_kernel<SRC>;
  static std::atomic<uint32_t> attribute_set{0};
  cudaError_t e = prepare_kernel(kernel, xe::cpb::kSmemBytes, attribute_set);
  if (e != cudaSuccess) return fail(XE_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", who, cudaGetErrorString(e));
  kernel<<<grid, xe::cpb::kThreads, xe::cpb::kSmemBytes, s>>>(q, mx1, mx2, my, mg);
  return check_launch(who);
}

// Shared by both entry points: src is xe::cpb::kDense / kDense2 (x1 = A, x2 = A2 or null, both
// (folds, m, 64)) or kGather2 (x1 = the (table_folds, states, 64) table).
xe_status cpb_run(const char* who, int src, const float* x1, const float* x2, int64_t table_folds, int64_t states,
                  const uint8_t* pixels, int64_t px_sm, int64_t px_sv, int64_t variables, const int32_t* var_of_fold,
                  int64_t fold_offset,
                  const float* y, const float* g, int64_t g_folds, const float* w, float* dx, float* dw, int64_t folds,
                  int64_t m, int32_t shift_mode, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (!x1 || !y || !g || !w || !dx || !dw) return fail(XE_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
  if (folds < 0 || m < 0) return fail(XE_ERR_INVALID_ARGUMENT, "%s: negative extent", who);
  if (g_folds < 1) return fail(XE_ERR_INVALID_ARGUMENT, "%s: g_folds must be positive", who);
  if (shift_mode != XE_SHIFT_MAX && shift_mode != XE_SHIFT_MIN)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: unknown shift mode %d", who, shift_mode);
  if (folds == 0) return XE_OK;
  if (m == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, (size_t)folds * 4096 * sizeof(float), s);
    if (e != cudaSuccess) return fail(XE_ERR_CUDA, "%s: %s", who, cudaGetErrorString(e));
    return XE_OK;
  }
  const CpbGeometry geo = cpb_geometry(folds, m);
  if (m > INT32_MAX || geo.num_tiles > INT32_MAX || g_folds > INT32_MAX)
    return fail(XE_ERR_NOT_SUPPORTED, "%s: too many rows", who);
  const size_t need = cpb_workspace_bytes(geo, folds);
  if (workspace_bytes < need || (need > 0 && !workspace))
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: workspace of %zu bytes, %zu needed", who, workspace_bytes, need);
  if (!aligned16(w) || !aligned16(dx))
    return fail(XE_ERR_NOT_SUPPORTED, "%s: operands must be contiguous and 16-byte aligned", who);
  CUtensorMap mx1{}, mx2{}, my{}, mg{};
  bool maps = encode_rows_map(&my, y, folds, m) && encode_rows_map(&mg, g, g_folds, m);
  if (src == xe::cpb::kGather2) {
    maps = maps && encode_gather_map(&mx1, x1, table_folds * states, 64, 64);
  } else {
    maps = maps && encode_rows_map(&mx1, x1, folds, m);
    if (x2) maps = maps && encode_rows_map(&mx2, x2, folds, m);
  }
  if (!maps) return fail(XE_ERR_NOT_SUPPORTED, "%s: operands must be contiguous and 16-byte aligned", who);
  xe::cpb::Params q{};
  q.w = w;
  q.dx = dx;
  q.folds = (int)folds;
  q.M = (int)m;
  q.tiles_m = (int)geo.tiles_m;
  q.num_tiles = (int)geo.num_tiles;
  q.g_folds = (int)g_folds;
  q.shift_min = shift_mode == XE_SHIFT_MIN ? 1 : 0;
  q.pieces = geo.pieces;
  q.partials = static_cast<float*>(workspace);
  q.table = src == xe::cpb::kGather2 ? x1 : nullptr;
  q.pixels = pixels;
  q.var = var_of_fold;
  q.px_sm = px_sm;
  q.px_sv = px_sv;
  q.variables = variables;
  q.states = (int)states;
  q.pair = (int)fold_offset;
  xe_status st;
  if (src == xe::cpb::kGather2) st = launch_cpb_t<xe::cpb::kGather2>(who, q, mx1, mx1, my, mg, geo.grid, s);
  else if (x2) st = launch_cpb_t<xe::cpb::kDense2>(who, q, mx1, mx2, my, mg, geo.grid, s);
  else st = launch_cpb_t<xe::cpb::kDense>(who, q, mx1, mx1, my, mg, geo.grid, s);
  if (st != XE_OK) return st;
  const int64_t threads = folds * 1024;
  xe::cpb::cpb_reduce_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
      q.partials, q.folds, q.pieces, q.tiles_m, q.num_tiles, geo.grid, dw);
  return check_launch(who);
}

}  // namespace

extern "C" {

size_t xe_cp_layer_backward_workspace_size(int64_t folds, int64_t m) {
  if (folds <= 0 || m <= 0) return 0;
  return cpb_workspace_bytes(cpb_geometry(folds, m), folds);
}

xe_status xe_cp_layer_backward(const float* a, const float* a2, const float* y, const float* g, int64_t g_folds,
                               const float* w, float* da, float* dw, int64_t folds, int64_t m, int32_t shift_mode,
                               void* workspace, size_t workspace_bytes, void* stream) {
  return cpb_run("xe_cp_layer_backward", a2 ? xe::cpb::kDense2 : xe::cpb::kDense, a, a2, 0, 0, nullptr, 0, 0, 0, nullptr, 0,
                 y, g, g_folds, w, da, dw, folds, m, shift_mode, workspace, workspace_bytes, as_stream(stream));
}

xe_status xe_cp_layer_backward_gather_pair(const float* table, int64_t table_folds, int64_t states,
                                           const uint8_t* pixels, int64_t pixel_sample_stride,
                                           int64_t pixel_var_stride, int64_t variables, const int32_t* var_of_fold,
                                           int64_t fold_offset, const float* y, const float* g, int64_t g_folds,
                                           const float* w, float* da, float* dw, int64_t folds, int64_t m,
                                           int32_t shift_mode, void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "xe_cp_layer_backward_gather_pair";
  if (!pixels) return fail(XE_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
  if (states < 1 || fold_offset < 1 || variables < 1 || pixel_sample_stride < 0 || pixel_var_stride < 0)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: states, fold_offset and variables must be positive, strides non-negative",
                who);
  if (table_folds < folds + fold_offset)
    return fail(XE_ERR_INVALID_ARGUMENT, "%s: the table has %lld folds, %lld needed", who, (long long)table_folds,
                (long long)(folds + fold_offset));
  if (table_folds * states * 64 > INT32_MAX) return fail(XE_ERR_NOT_SUPPORTED, "%s: table too large", who);
  return cpb_run(who, xe::cpb::kGather2, table, nullptr, table_folds, states, pixels, pixel_sample_stride,
                 pixel_var_stride, variables, var_of_fold, fold_offset, y, g, g_folds, w, da, dw, folds, m, shift_mode, workspace, workspace_bytes,
                 as_stream(stream));
}

xe_status xe_state_table_pair_grad(const float* da, int64_t folds, int64_t m, const uint8_t* pixels,
                                   int64_t pixel_sample_stride, int64_t pixel_var_stride, int64_t variables,
                                   const int32_t* var_of_fold, int64_t fold_offset, int64_t states,
                                   float* table_grad, void* stream) {
  const char* who = "xe_state_table_pair_grad";
  if (!da || !pixels || !table_grad) return fail(XE_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
  if (folds < 0 || m < 0) return fail(XE_ERR_INVALID_ARGUMENT, "%s: negative extent", who);
  if (states < 1 || states > 256 || fold_offset < 1 || variables < 1 || pixel_sample_stride < 0 || pixel_var_stride < 0)
    return fail(states > 256 ? XE_ERR_NOT_SUPPORTED : XE_ERR_INVALID_ARGUMENT,
                "%s: needs 1 <= states <= 256, positive fold_offset and variables, non-negative strides", who);
  if (m > INT32_MAX || folds + fold_offset > INT32_MAX) return fail(XE_ERR_NOT_SUPPORTED, "%s: too many rows", who);
  if (!aligned16(da) || !aligned16(table_grad)) return fail(XE_ERR_NOT_SUPPORTED, "%s: 16-byte aligned buffers", who);
  if (folds == 0) return XE_OK;
  static std::atomic<uint32_t> attribute_set{0};
  cudaError_t e = prepare_kernel(xe::cpb::table_grad_pair_kernel, xe::cpb::kTgSmemBytes, attribute_set);
  if (e != cudaSuccess) return fail(XE_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", who, cudaGetErrorString(e));
  const int grid = (int)std::min<int64_t>(folds, current_device_sms());
  xe::cpb::table_grad_pair_kernel<<<grid, xe::cpb::kTgThreads, xe::cpb::kTgSmemBytes, as_stream(stream)>>>(
      da, (int)folds, (int)m, pixels, pixel_sample_stride, pixel_var_stride, variables, var_of_fold, (int)fold_offset,
      (int)states, table_grad);
  return check_launch(who);
}

}  // extern "C"

extern "C" {

xe_status xe_u8_transpose(const uint8_t* x, int64_t rows, int64_t cols, int64_t row_stride, uint8_t* y, void* stream) {
  if (!x || !y) return fail(XE_ERR_INVALID_ARGUMENT, "xe_u8_transpose: null pointer");
  if (rows < 0 || cols < 0 || row_stride < cols) return fail(XE_ERR_INVALID_ARGUMENT, "xe_u8_transpose: bad extents");
  if (rows == 0 || cols == 0) return XE_OK;
  const int64_t gx = (cols + 31) / 32, gy = (rows + 31) / 32;
  if (gx > INT32_MAX || gy > 65535) return fail(XE_ERR_NOT_SUPPORTED, "xe_u8_transpose: too many rows");
  xe::transpose_u8<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, as_stream(stream)>>>(x, rows, cols, row_stride, y);
  return check_launch("xe_u8_transpose");
}

}  // extern "C"
