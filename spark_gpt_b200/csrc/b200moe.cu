// C-ABI entry points of libb200moe.so (declared in include/b200moe.h):
// argument checks, TMA tensor-map construction, launch shapes.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/b200moe.h"
#include "grouped_gemm.cuh"
#include "grouped_gemm_2sm.cuh"
#include "routing.cuh"
#include "ep.cuh"
#include "muon.cuh"
#include "fp8.cuh"

namespace b200moe {
namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return B200MOE_OK;
}

#define REQUIRE(cond, ...)                                    \
  do {                                                        \
    if (!(cond)) return fail(B200MOE_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// SMs the persistent kernels (expert GEMMs, row reductions) size their grids
// for: all of them, or fewer while a collective runs beside them on another
// stream (b200moe_set_persistent_sm_limit), so that every CTA of the grid is
// resident at once and no statically scheduled tile waits for the collective.
int g_sm_limit = 0;

// SMs' worth of blocks the peer-memory transfer kernels launch (0 = a grid
// over every SM): set while a transfer runs on a copy stream beside the
// compute stream, so that the compute stream's kernels keep their SMs.
int g_transfer_sm_limit = 0;

int persistent_sms() {
  const int n = num_sms();
  return (g_sm_limit > 0 && g_sm_limit < n) ? g_sm_limit : n;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major (outer, inner) matrix with row stride
// `ld` elements; box (box_inner, box_outer) with the 128-byte swizzle.
int make_tmap(CUtensorMap* m, const void* base, long long inner, long long outer, long long ld,
              int box_inner, int box_outer, const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: base pointer not 16-byte aligned", what);
  if ((ld * 2) % 16 != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: row stride not a multiple of 16 bytes", what);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

// 2-D fp8 (one byte per element) tensor map with the 128-byte swizzle: a
// K-major box of 128 elements x box_outer rows, or an MN-major box of
// 128 x 128.
int make_tmap_u8(CUtensorMap* m, const void* base, long long inner, long long outer,
                 long long ld, int box_inner, int box_outer, const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: base pointer not 16-byte aligned", what);
  if (ld % 16 != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: row stride not a multiple of 16 bytes", what);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

// Tensor map for row gathers (tile::gather4) from a token-major (rows, cols)
// bf16 matrix: box of one row by 64 columns.
int make_gather_tmap(CUtensorMap* m, const void* base, long long cols, long long rows,
                     const char* what) {
  return make_tmap(m, base, cols, rows, cols, 64, 1, what);
}

template <int BN>
constexpr int stages_for() {
  return BN == 256 ? 4 : (BN == 128 ? 6 : 8);
}

template <int BN, bool A_MN, bool B_MN, int EPI, int SCHED, int GATHER = kGatherNone>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                cudaStream_t st, const char* what) {
  constexpr int STAGES = stages_for<BN>();
  auto kern = grouped_gemm_kernel<BN, A_MN, B_MN, EPI, SCHED, STAGES, GATHER>;
  const int smem = static_cast<int>(GemmSmem<BN, STAGES>::kTotal);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  kern<<<persistent_sms(), kGemmThreads, smem, st>>>(ta, tb, p);
  return check_launch(what);
}

// Operand ring depth of the pair kernel: as many stages as fit next to the
// output staging ring in the 227 KB a CTA may hold (deeper rings hide more of
// the operand load latency), at most B200MOE_PAIR_STAGES_MAX.
#ifndef B200MOE_PAIR_STAGES_MAX
#define B200MOE_PAIR_STAGES_MAX 8
#endif
constexpr uint32_t kMaxDynSmem = 227 * 1024;
constexpr int kMaxWgradSegments = 64;  // row segments of one segmented weight gradient

template <int BN, bool TMA_OUT, bool GU_IN = false>
constexpr int pair_stages() {
  using S1 = PairSmem<BN, 1, TMA_OUT, GU_IN>;
  constexpr int fit = static_cast<int>((kMaxDynSmem - (S1::kTotal - S1::kStageBytes)) /
                                       S1::kStageBytes);
  return fit < B200MOE_PAIR_STAGES_MAX ? fit : B200MOE_PAIR_STAGES_MAX;
}

// Expert GEMMs run as two-CTA pair tiles when the shape allows (switchable for
// parity tests of the two kernels against each other).
int g_pair_gemm = 1;

template <int BN, bool A_MN, bool B_MN, int EPI, int SCHED, int OP = kOpBf16>
int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to0,
                     const CUtensorMap& to1, const GemmParams& p, cudaStream_t st,
                     const char* what) {
  constexpr bool kTmaOut = TmaOut<EPI>::value;
  constexpr bool kGuIn = GuIn<EPI>::value;
  constexpr int STAGES = pair_stages<BN, kTmaOut, kGuIn>();
  auto kern = grouped_gemm_pair_kernel<BN, A_MN, B_MN, EPI, SCHED, STAGES, OP>;
  const int smem = static_cast<int>(PairSmem<BN, STAGES, kTmaOut, kGuIn>::kTotal);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(persistent_sms() & ~1), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, to0, to1, p);
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

// Whether an expert GEMM runs as two-CTA pair tiles: BN of 128/256, E <= 256
// (the kernel's per-expert pair table) and, for weight gradients, M a
// multiple of 256.  Tensor maps of K-major B depend on it (box of BN/2 rows
// per CTA instead of BN).
bool use_pair(int BN, int sched, int num_groups, int m_tiles) {
  return g_pair_gemm && BN >= 128 && num_groups <= kMaxPairExperts &&
         (sched == kRowsRagged || m_tiles % 2 == 0);
}

// Output tensor maps of the pair kernel's TMA-store epilogue: a {32, 32} box
// with the 64-byte swizzle over a (rows, cols) bf16 matrix.
int make_out_tmap(CUtensorMap* m, const void* base, long long cols, long long rows,
                  const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

// Output tensor maps of the plain bf16-store epilogue (kEpiStoreBf16): the
// {32, 32} box above, or a {64, 32} box with the 128-byte swizzle when that
// epilogue stores two TMEM chunks per box.
int make_store_tmap(CUtensorMap* m, const void* base, long long cols, long long rows,
                    const char* what) {
  if (!kWideBf16Store) return make_out_tmap(m, base, cols, rows, what);
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

// Output tensor maps of the fp32 TMA-store epilogue: a {16, 32} box (64 bytes
// of fp32 per row) with the 64-byte swizzle over a (rows, cols) fp32 matrix.
int make_out_tmap_f32(CUtensorMap* m, const void* base, long long cols, long long rows,
                      const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 4)};
  cuuint32_t box[2] = {16, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

// Output tensor maps of the weight-gradient epilogue (kEpiStoreF32Tma): the
// {16, 32} box above, or a {32, 32} box with the 128-byte swizzle when that
// epilogue stores a whole TMEM chunk per box.
int make_wgrad_tmap(CUtensorMap* m, const void* base, long long cols, long long rows,
                    const char* what) {
  if (!kWideF32Store) return make_out_tmap_f32(m, base, cols, rows, what);
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

// Output tensor maps of the fp8 TMA-store epilogues: a {32, 32} box of bytes,
// unswizzled, over a (rows, cols) fp8 matrix.
int make_out_tmap_u8(CUtensorMap* m, const void* base, long long cols, long long rows,
                     const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || cols % 16 != 0)
    return fail(B200MOE_ERR_INVALID_ARG, "%s: base or row stride not 16-byte aligned", what);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200MOE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return B200MOE_OK;
}

template <int BN, bool A_MN, bool B_MN, int EPI, int SCHED>
int launch_expert_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                       cudaStream_t st, const char* what, const CUtensorMap* to0 = nullptr,
                       const CUtensorMap* to1 = nullptr) {
  if constexpr (BN >= 128) {
    if (use_pair(BN, SCHED, p.num_groups, p.m_tiles) &&
        (SCHED == kKRagged || p.pad_offsets != nullptr)) {
      if (TmaOut<EPI>::value && p.scatter_rows == nullptr && to0 == nullptr)
        return fail(B200MOE_ERR_INVALID_ARG, "%s: missing output tensor map", what);
      return launch_gemm_pair<BN, A_MN, B_MN, EPI, SCHED>(ta, tb, to0 ? *to0 : ta,
                                                         to1 ? *to1 : (to0 ? *to0 : ta), p, st,
                                                         what);
    }
  }
  return launch_gemm<BN, A_MN, B_MN, EPI, SCHED>(ta, tb, p, st, what);
}

GemmParams blank_params() {
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  return p;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int grid_for(long long items, int per_block) {
  long long g = (items + per_block - 1) / per_block;
  const long long cap = static_cast<long long>(num_sms()) * 32;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// Grid of a transfer kernel (grid-stride warps over rows): at most 8 blocks of
// 256 threads per SM of the transfer SM limit, when one is set.
int transfer_grid(long long items, int per_block) {
  const int g = grid_for(items, per_block);
  return g_transfer_sm_limit > 0 ? std::min(g, g_transfer_sm_limit * 8) : g;
}

// lanes per token of the router kernels: 8 logits per lane, so 8*L >= width
int lanes_for(long long width) {
  int l = 2;
  while (l < 32 && 8 * l < width) l *= 2;
  return l;
}

#define B200_SWITCH_LANES(width, ...)          \
  switch (lanes_for(width)) {                  \
    case 2: { constexpr int L = 2; __VA_ARGS__ } break;   \
    case 4: { constexpr int L = 4; __VA_ARGS__ } break;   \
    case 8: { constexpr int L = 8; __VA_ARGS__ } break;   \
    case 16: { constexpr int L = 16; __VA_ARGS__ } break; \
    default: { constexpr int L = 32; __VA_ARGS__ } break; \
  }

// Launch the shared-memory row reduction (combine forward / gather backward).
// Returns -1 when one token's k rows do not fit a ring slot (caller falls back).
constexpr int kReduceSmemPerBlock = 72 * 1024;  // three blocks per SM

// Blocks of the row reduction: three per SM (kReduceSmemPerBlock), at most T.
long long row_reduce_blocks(long long T, int sms) {
  return std::min<long long>(3LL * sms, std::max<long long>(T, 1));
}

int launch_row_reduce(const __nv_bfloat16* rows, const int* inv_pad,
                      const __nv_bfloat16* weights, const __nv_bfloat16* addend, long long T,
                      int k, int H, __nv_bfloat16* out, cudaStream_t st, const char* what,
                      bool partial, const NormBwd* norm = nullptr, long long* grid_out = nullptr) {
  const long long slot_bytes = 2LL * H * k;
  // slots: a multiple of the consumer-group count, at least one per group
  const int min_slots = kReduceGroups;
  if (slot_bytes * min_slots > kReduceSmemPerBlock || H % (8 * kReduceWarpsPerToken) != 0 ||
      k > kMaxTopK)
    return -1;
  // vectors per lane of the fused norm backward: one per 1024 columns
  const int nv = norm ? (H + 1023) / 1024 : 0;
  if (nv > kNormVecsMax) return -1;
  int slots = kMaxReduceSlots;
  while (slots > min_slots && slots * slot_bytes > kReduceSmemPerBlock) slots -= kReduceGroups;
  const size_t smem = static_cast<size_t>(slots) * slot_bytes + 2 * slots * sizeof(uint64_t);
  const bool skip = partial && inv_pad;
  decltype(&row_reduce_kernel<false, 0>) kern;
  switch (nv) {
    case 0: kern = skip ? row_reduce_kernel<true, 0> : row_reduce_kernel<false, 0>; break;
    case 1: kern = skip ? row_reduce_kernel<true, 1> : row_reduce_kernel<false, 1>; break;
    case 2: kern = skip ? row_reduce_kernel<true, 2> : row_reduce_kernel<false, 2>; break;
    default: kern = skip ? row_reduce_kernel<true, 4> : row_reduce_kernel<false, 4>; break;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  // resident blocks per SM: three (the plain reduction and H <= 1024), fewer
  // when the fused norm backward holds more columns per lane
  const int per_sm = nv <= 1 ? 3 : (nv == 2 ? 2 : 1);
  const long long grid = std::min<long long>(row_reduce_blocks(T, persistent_sms()),
                                             static_cast<long long>(per_sm) * persistent_sms());
  if (grid_out) *grid_out = grid;
  kern<<<static_cast<int>(grid), kReduceThreads, smem, st>>>(rows, inv_pad, weights, addend, T, k,
                                                              H, slots, out,
                                                              norm ? *norm : NormBwd{});
  return check_launch(what);
}

}  // namespace
}  // namespace b200moe

using namespace b200moe;

extern "C" {

int b200moe_version(void) { return 100; }

int b200moe_set_persistent_sm_limit(int sms) {
  const int prev = g_sm_limit;
  g_sm_limit = sms > 0 ? (sms < 2 ? 2 : sms) : 0;
  return prev;
}

int b200moe_set_transfer_sm_limit(int sms) {
  const int prev = g_transfer_sm_limit;
  g_transfer_sm_limit = sms > 0 ? sms : 0;
  return prev;
}

int b200moe_set_pair_gemm(int enable) {
  const int prev = g_pair_gemm;
  g_pair_gemm = enable ? 1 : 0;
  return prev;
}

const char* b200moe_last_error(void) { return t_last_error.c_str(); }

int b200moe_fault_read_and_clear(unsigned int* fault) {
  REQUIRE(fault, "fault: null pointer");
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_fault, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_fault, &zero, sizeof(zero));
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "fault read: %s", cudaGetErrorString(e));
  *fault = v;
  return B200MOE_OK;
}

int b200moe_fault_snapshot(unsigned int* dst, void* stream) {
  REQUIRE(dst, "fault_snapshot: null pointer");
  cudaError_t e = cudaMemcpyFromSymbolAsync(dst, g_fault, sizeof(unsigned int), 0,
                                            cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "fault snapshot: %s", cudaGetErrorString(e));
  return B200MOE_OK;
}

long long b200moe_padded_rows(long long routed_rows, int num_experts) {
  const long long r = routed_rows + static_cast<long long>(num_experts) * (kRowTile - 1);
  return (r + kRowTile - 1) / kRowTile * kRowTile;
}

int b200moe_router_width(int num_experts) {
  if (num_experts <= 64) return 64;
  if (num_experts <= 128) return 128;
  return 256;
}

int b200moe_cast_f32_to_bf16(const float* src, long long rows_in, long long cols,
                             long long rows_out, void* dst, void* stream) {
  REQUIRE(src && dst, "cast: null pointer");
  REQUIRE(rows_in >= 0 && rows_out >= rows_in && cols > 0, "cast: bad shape");
  REQUIRE((rows_out * cols) % 4 == 0, "cast: rows_out*cols must be a multiple of 4");
  REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0 && reinterpret_cast<uintptr_t>(dst) % 8 == 0,
          "cast: misaligned pointer");
  const long long n4 = rows_out * cols / 4;
  cast_f32_bf16_kernel<<<grid_for(n4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, rows_in, cols, rows_out, static_cast<__nv_bfloat16*>(dst));
  return check_launch("cast_f32_to_bf16");
}

// ---------------------------------------------------------------- router
int b200moe_router_logits(const void* x, const void* w, long long T, int H, int W, void* logits,
                          void* stream) {
  REQUIRE(x && w && logits, "router_logits: null pointer");
  REQUIRE(T > 0 && H % 64 == 0 && H > 0, "router_logits: H must be a positive multiple of 64");
  REQUIRE(W == 64 || W == 128 || W == 256, "router_logits: width must be 64, 128 or 256");
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, x, H, T, H, 64, 128, "router_logits x"))) return rc;
  if ((rc = make_tmap(&tb, w, H, W, H, 64, W, "router_logits w"))) return rc;
  GemmParams p = blank_params();
  p.num_groups = 1;
  p.m_tiles = static_cast<int>((T + 127) / 128);
  p.n_tiles = 1;
  p.k_blocks = H / 64;
  p.m_valid = T;
  p.n_valid = W;
  p.out = logits;
  p.ld_out = W;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (W) {
    case 64: return launch_gemm<64, false, false, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "router_logits");
    case 128: return launch_gemm<128, false, false, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "router_logits");
    default: return launch_gemm<256, false, false, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "router_logits");
  }
}

int b200moe_router_topk_fwd(const void* logits, int logits_f32, long long ld, long long T, int E,
                            int k, int norm, long long* selected, void* weights, void* stream) {
  REQUIRE(logits && selected && weights, "router_topk_fwd: null pointer");
  REQUIRE(E >= 1 && E <= 256 && ld >= E && ld <= 256, "router_topk_fwd: need 1 <= E <= ld <= 256");
  REQUIRE(k >= 1 && k <= kMaxTopK && k <= E, "router_topk_fwd: need 1 <= k <= min(E, 16)");
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* w = static_cast<__nv_bfloat16*>(weights);
  const int vec = aligned16(logits) && (ld * (logits_f32 ? 4 : 2)) % 16 == 0;
  B200_SWITCH_LANES(E, {
    const int grid = grid_for(T, 256 / L);
    if (logits_f32) {
      if (k <= 8)
        router_topk_fwd_kernel<L, 8, float><<<grid, 256, 0, st>>>(
            static_cast<const float*>(logits), ld, T, E, k, norm, vec, selected, w);
      else
        router_topk_fwd_kernel<L, kMaxTopK, float><<<grid, 256, 0, st>>>(
            static_cast<const float*>(logits), ld, T, E, k, norm, vec, selected, w);
    } else {
      if (k <= 8)
        router_topk_fwd_kernel<L, 8, __nv_bfloat16><<<grid, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(logits), ld, T, E, k, norm, vec, selected, w);
      else
        router_topk_fwd_kernel<L, kMaxTopK, __nv_bfloat16><<<grid, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(logits), ld, T, E, k, norm, vec, selected, w);
    }
  })
  return check_launch("router_topk_fwd");
}

int b200moe_router_topk_bwd(const void* logits, long long ld, const long long* selected,
                            const float* d_weights, const void* d_extra, long long T, int E, int k,
                            int norm, void* d_logits, void* stream) {
  REQUIRE(logits && selected && d_weights && d_logits, "router_topk_bwd: null pointer");
  REQUIRE(E >= 1 && E <= 256 && ld >= E && ld <= 256, "router_topk_bwd: need 1 <= E <= ld <= 256");
  REQUIRE(k >= 1 && k <= kMaxTopK && k <= E, "router_topk_bwd: need 1 <= k <= min(E, 16)");
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* lg = static_cast<const __nv_bfloat16*>(logits);
  auto* ex = static_cast<const __nv_bfloat16*>(d_extra);
  auto* out = static_cast<__nv_bfloat16*>(d_logits);
  const int vec = aligned16(lg) && aligned16(out) && (ex == nullptr || aligned16(ex)) &&
                  (ld * 2) % 16 == 0;
  B200_SWITCH_LANES(ld, {
    if (k <= 8)
      router_topk_bwd_kernel<L, 8><<<grid_for(T, 256 / L), 256, 0, st>>>(
          lg, ld, selected, d_weights, ex, T, E, k, norm, vec, out);
    else
      router_topk_bwd_kernel<L, kMaxTopK><<<grid_for(T, 256 / L), 256, 0, st>>>(
          lg, ld, selected, d_weights, ex, T, E, k, norm, vec, out);
  })
  return check_launch("router_topk_bwd");
}

int b200moe_router_dgrad(const void* d_logits, const void* w, long long T, int H, int W, void* dx,
                         void* stream) {
  REQUIRE(d_logits && w && dx, "router_dgrad: null pointer");
  REQUIRE(T > 0 && H % 128 == 0, "router_dgrad: H must be a multiple of 128");
  REQUIRE(W == 64 || W == 128 || W == 256, "router_dgrad: width must be 64, 128 or 256");
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, d_logits, W, T, W, 64, 128, "router_dgrad d_logits"))) return rc;
  if ((rc = make_tmap(&tb, w, H, W, H, 64, 64, "router_dgrad w"))) return rc;
  GemmParams p = blank_params();
  p.num_groups = 1;
  p.m_tiles = static_cast<int>((T + 127) / 128);
  const int BN = (H % 256 == 0) ? 256 : 128;
  p.n_tiles = H / BN;
  p.k_blocks = W / 64;
  p.b_group_rows = 0;
  p.m_valid = T;
  p.n_valid = H;
  p.out = dx;
  p.ld_out = H;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 256 && g_pair_gemm) {
    // K = W is one or a few 64-column blocks, so the tile's time is its epilogue: the
    // two-CTA kernel writes it through shared memory with TMA stores (rows >= T are
    // clipped by the tensor map; the rows of the tile past T load as zeros)
    CUtensorMap to;
    if ((rc = make_store_tmap(&to, dx, H, T, "router_dgrad dx"))) return rc;
    return launch_gemm_pair<256, false, true, kEpiStoreBf16, kRowsRagged>(ta, tb, to, to, p, st,
                                                                          "router_dgrad");
  }
  if (BN == 256) return launch_gemm<256, false, true, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "router_dgrad");
  return launch_gemm<128, false, true, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "router_dgrad");
}

namespace {
// K splits of the router weight gradient: enough (split, 128-row M tile) work items for
// about two per SM.
void router_wgrad_splits(long long T, int H, int* splits, int* blocks_per_split) {
  const int kb = static_cast<int>((T + 63) / 64);
  const int m_tiles = H / 128;
  int s = (2 * num_sms() + m_tiles - 1) / m_tiles;
  s = s < 1 ? 1 : (s > kb ? kb : s);
  const int per = (kb + s - 1) / s;
  *blocks_per_split = per;
  *splits = (kb + per - 1) / per;
}
}  // namespace

long long b200moe_router_wgrad_scratch_bytes(long long T, int H, int E) {
  int s = 1, per = 1;
  if (T <= 0 || H < 128) return 0;
  router_wgrad_splits(T, H, &s, &per);
  return static_cast<long long>(s) * E * H * static_cast<long long>(sizeof(float));
}

int b200moe_router_wgrad(const void* x, const void* d_logits, long long T, int H, int E, int W,
                         float* dw, int accumulate, void* scratch, long long scratch_bytes,
                         void* stream) {
  REQUIRE(x && d_logits && dw && scratch, "router_wgrad: null pointer");
  REQUIRE(T > 0 && H % 128 == 0, "router_wgrad: H must be a multiple of 128");
  REQUIRE(W == 64 || W == 128 || W == 256, "router_wgrad: width must be 64, 128 or 256");
  REQUIRE(E >= 1 && E <= W, "router_wgrad: need 1 <= E <= width");
  REQUIRE(T <= 0x7fffffffLL, "router_wgrad: too many tokens");
  REQUIRE(scratch_bytes >= b200moe_router_wgrad_scratch_bytes(T, H, E),
          "router_wgrad: scratch too small");
  int splits = 1, per = 1;
  router_wgrad_splits(T, H, &splits, &per);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, x, H, T, H, 64, 64, "router_wgrad x"))) return rc;
  if ((rc = make_tmap(&tb, d_logits, W, T, W, 64, 64, "router_wgrad d_logits"))) return rc;
  GemmParams p = blank_params();
  p.num_groups = splits;
  p.m_tiles = H / 128;
  p.n_tiles = 1;
  p.k_blocks = static_cast<int>((T + 63) / 64);
  p.k_split_blocks = per;
  p.n_valid = E;
  p.out = scratch;
  p.ld_out = H;
  p.out_group_stride = static_cast<long long>(E) * H;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (W) {
    case 64: rc = launch_gemm<64, true, true, kEpiStoreF32T, kKRagged>(ta, tb, p, st, "router_wgrad"); break;
    case 128: rc = launch_gemm<128, true, true, kEpiStoreF32T, kKRagged>(ta, tb, p, st, "router_wgrad"); break;
    default: rc = launch_gemm<256, true, true, kEpiStoreF32T, kKRagged>(ta, tb, p, st, "router_wgrad"); break;
  }
  if (rc) return rc;
  const long long n = static_cast<long long>(E) * H;
  reduce_splits_kernel<<<grid_for(n / 4, 256), 256, 0, st>>>(static_cast<const float*>(scratch),
                                                             splits, n, dw, accumulate);
  return check_launch("router_wgrad reduce");
}

// ---------------------------------------------------------------- dispatch
long long b200moe_dispatch_scratch_bytes(long long T, int k, int E) {
  const long long R = T * k;
  const long long nblk = (R + kDispatchChunk - 1) / kDispatchChunk;
  return (nblk > 0 ? nblk : 1) * E * static_cast<long long>(sizeof(int));
}

}  // extern "C"

namespace {

// count -> scan -> scatter over nblk chunks of kDispatchChunk slots; `base`
// holds nblk * E ints.
template <int WARPS>
int launch_dispatch_scatter(const long long* selected, long long R, int E, int nblk,
                            const int* base, int* row_flat, int* inv_pad, cudaStream_t st,
                            const char* tag) {
  const size_t shm = static_cast<size_t>(WARPS) * E * sizeof(int);
  if (shm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(dispatch_scatter_kernel<WARPS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm);
    if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "%s scatter: %s", tag, cudaGetErrorString(e));
  }
  dispatch_scatter_kernel<WARPS><<<nblk, WARPS * 32, shm, st>>>(selected, R, E, nblk, base,
                                                                row_flat, inv_pad);
  return check_launch(tag);
}

int launch_dispatch(const long long* selected, long long R, int E, int nblk, int* base,
                    int* counts, int* offsets, int* pad_offsets, int* row_flat, int* inv_pad,
                    int* tile_expert, cudaStream_t st, const char* tag) {
  dispatch_count_kernel<<<nblk, kDispatchThreads, E * sizeof(int), st>>>(selected, R, E, nblk, base);
  int rc = check_launch(tag);
  if (rc) return rc;
  dispatch_scan_kernel<<<1, 1024, (2 * E + 1) * sizeof(int), st>>>(base, nblk, E, counts, offsets,
                                                                   pad_offsets, row_flat, tile_expert);
  if ((rc = check_launch(tag))) return rc;
  // 32 warps per chunk while their expert tables fit (E <= 1024: 128 KB), else 8
  return E <= 1024 ? launch_dispatch_scatter<32>(selected, R, E, nblk, base, row_flat, inv_pad, st, tag)
                   : launch_dispatch_scatter<8>(selected, R, E, nblk, base, row_flat, inv_pad, st, tag);
}

}  // namespace

extern "C" {

int b200moe_dispatch(const long long* selected, long long T, int k, int E, int* counts,
                     int* offsets, int* pad_offsets, int* row_flat, int* inv_pad, int* tile_expert,
                     void* scratch, long long scratch_bytes, void* stream) {
  REQUIRE(selected && counts && offsets && pad_offsets && row_flat && inv_pad && tile_expert &&
              scratch,
          "dispatch: null pointer");
  REQUIRE(E >= 1 && E <= 4096 && k >= 1 && k <= E, "dispatch: need 1 <= k <= E <= 4096");
  const long long R = T * k;
  REQUIRE(R >= 0 && b200moe_padded_rows(R, E) < 0x7fffffffLL, "dispatch: too many rows");
  REQUIRE(scratch_bytes >= b200moe_dispatch_scratch_bytes(T, k, E), "dispatch: scratch too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nblk = static_cast<int>(R > 0 ? (R + kDispatchChunk - 1) / kDispatchChunk : 1);
  return launch_dispatch(selected, R, E, nblk, static_cast<int*>(scratch), counts, offsets,
                         pad_offsets, row_flat, inv_pad, tile_expert, st, "dispatch");
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free dispatch
// Per-(expert, 4096-slot chunk) row counts of b200moe_dispatch_noalloc live in this fixed
// device array instead of caller-provided scratch.  1 MiB; every GPU that loads the library
// keeps it until the process exits.  Host code must not pass the array's name to a kernel
// (on the host it is only a stand-in, not a device address): its device address is looked
// up once per device with cudaGetSymbolAddress and cached until exit (a device reset after
// the first call is not supported: the cached address belongs to the old context).
namespace {
constexpr long long kNoAllocDispatchInts = 262144;
static __device__ __align__(256) int g_noalloc_dispatch_counts[kNoAllocDispatchInts];

std::mutex g_noalloc_mu;
int* g_noalloc_ptr[64] = {nullptr};

int noalloc_dispatch_scratch(int** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "dispatch_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(B200MOE_ERR_UNSUPPORTED, "dispatch_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_dispatch_counts);
    if (e != cudaSuccess)
      return fail(B200MOE_ERR_CUDA, "dispatch_noalloc: cudaGetSymbolAddress: %s",
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<int*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return B200MOE_OK;
}
}  // namespace

extern "C" {

int b200moe_dispatch_noalloc(const long long* selected, long long T, int k, int E, int* counts,
                             int* offsets, int* pad_offsets, int* row_flat, int* inv_pad,
                             int* tile_expert, void* stream) {
  REQUIRE(selected && counts && offsets && pad_offsets && row_flat && inv_pad && tile_expert,
          "dispatch_noalloc: null pointer");
  REQUIRE(E >= 1 && E <= 4096 && k >= 1 && k <= E, "dispatch_noalloc: need 1 <= k <= E <= 4096");
  const long long R = T * k;
  REQUIRE(R >= 0 && b200moe_padded_rows(R, E) < 0x7fffffffLL, "dispatch_noalloc: too many rows");
  const long long nblk_ll = R > 0 ? (R + kDispatchChunk - 1) / kDispatchChunk : 1;
  REQUIRE(nblk_ll * E <= kNoAllocDispatchInts,
          "dispatch_noalloc: T*k = %lld slots with E = %d experts needs %lld scratch counts "
          "(ceil(T*k/4096) * E); the built-in scratch holds %lld. Use b200moe_dispatch with "
          "caller-provided scratch for this size",
          R, E, nblk_ll * E, kNoAllocDispatchInts);
  int* base = nullptr;
  int rc = noalloc_dispatch_scratch(&base);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nblk = static_cast<int>(nblk_ll);
  // the count kernel writes every one of the nblk*E entries before the scan reads them, so
  // whatever an earlier call left in the array needs no clearing
  return launch_dispatch(selected, R, E, nblk, base, counts, offsets, pad_offsets, row_flat,
                         inv_pad, tile_expert, st, "dispatch_noalloc");
}

// ---------------------------------------------------------------- gather / combine
#ifndef B200MOE_TOKEN_ORDER
#define B200MOE_TOKEN_ORDER 1  // gather / combine backward traverse tokens (0: padded rows)
#endif

int b200moe_gather_rows(const void* x, const int* row_flat, const int* inv_pad,
                        const int* pad_offsets, long long T, int E, int k, int H,
                        long long rows_cap, void* xs, void* stream) {
  REQUIRE(x && row_flat && pad_offsets && xs, "gather_rows: null pointer");
  REQUIRE(H % 8 == 0 && H > 0 && k >= 1, "gather_rows: H must be a multiple of 8");
  auto* xp = static_cast<const __nv_bfloat16*>(x);
  auto* xsp = static_cast<__nv_bfloat16*>(xs);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B200MOE_TOKEN_ORDER && inv_pad) {
    REQUIRE(k <= 32 && T >= 0, "gather_rows: need k <= 32");
    const int grid = grid_for(T > rows_cap / 32 ? T : rows_cap / 32, 8);
    const int* tot = pad_offsets + E;
    switch (H) {
      case 256: scatter_rows_kernel<1><<<grid, 256, 0, st>>>(xp, inv_pad, row_flat, tot, T, k, H, xsp); break;
      case 512: scatter_rows_kernel<2><<<grid, 256, 0, st>>>(xp, inv_pad, row_flat, tot, T, k, H, xsp); break;
      case 1024: scatter_rows_kernel<4><<<grid, 256, 0, st>>>(xp, inv_pad, row_flat, tot, T, k, H, xsp); break;
      case 2048: scatter_rows_kernel<8><<<grid, 256, 0, st>>>(xp, inv_pad, row_flat, tot, T, k, H, xsp); break;
      default: scatter_rows_kernel<0><<<grid, 256, 0, st>>>(xp, inv_pad, row_flat, tot, T, k, H, xsp); break;
    }
    return check_launch("gather_rows");
  }
  const int grid = grid_for(rows_cap, 8);
  switch (H) {
    case 256: gather_rows_kernel<1><<<grid, 256, 0, st>>>(xp, row_flat, pad_offsets + E, k, H, xsp); break;
    case 512: gather_rows_kernel<2><<<grid, 256, 0, st>>>(xp, row_flat, pad_offsets + E, k, H, xsp); break;
    case 1024: gather_rows_kernel<4><<<grid, 256, 0, st>>>(xp, row_flat, pad_offsets + E, k, H, xsp); break;
    case 2048: gather_rows_kernel<8><<<grid, 256, 0, st>>>(xp, row_flat, pad_offsets + E, k, H, xsp); break;
    default: gather_rows_kernel<0><<<grid, 256, 0, st>>>(xp, row_flat, pad_offsets + E, k, H, xsp); break;
  }
  return check_launch("gather_rows");
}

int b200moe_gather_rows_bwd(const void* dxs, const int* inv_pad, const void* addend, long long T,
                            int k, int H, int partial, void* dx, void* stream) {
  REQUIRE(dxs && dx, "gather_rows_bwd: null pointer");
  REQUIRE(H % 8 == 0 && H > 0 && k >= 1 && k <= kMaxTopK, "gather_rows_bwd: bad shape");
  if (T == 0) return B200MOE_OK;
  {
    const int rc = launch_row_reduce(static_cast<const __nv_bfloat16*>(dxs), inv_pad, nullptr,
                                     static_cast<const __nv_bfloat16*>(addend), T, k, H,
                                     static_cast<__nv_bfloat16*>(dx),
                                     static_cast<cudaStream_t>(stream), "gather_rows_bwd",
                                     partial != 0);
    if (rc >= 0) return rc;
  }
  gather_rows_bwd_kernel<<<grid_for(T, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(dxs), inv_pad, static_cast<const __nv_bfloat16*>(addend), T,
      k, H, static_cast<__nv_bfloat16*>(dx));
  return check_launch("gather_rows_bwd");
}

int b200moe_rmsnorm_fwd(const void* x, const float* w, long long T, int H, float eps, void* x_n,
                        float* rstd, void* stream) {
  REQUIRE(x && w && x_n && rstd, "rmsnorm_fwd: null pointer");
  REQUIRE(H % 8 == 0 && H > 0, "rmsnorm_fwd: H must be a positive multiple of 8");
  REQUIRE(aligned16(x) && aligned16(x_n), "rmsnorm_fwd: x and x_n must be 16-byte aligned");
  if (T == 0) return B200MOE_OK;
  rmsnorm_fwd_kernel<<<grid_for(T, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), w, T, H, eps, static_cast<__nv_bfloat16*>(x_n), rstd);
  return check_launch("rmsnorm_fwd");
}

long long b200moe_gather_rows_bwd_rmsnorm_scratch_bytes(long long T, int H) {
  return row_reduce_blocks(T, num_sms()) * kReduceGroups * static_cast<long long>(H) *
         static_cast<long long>(sizeof(float));
}

int b200moe_gather_rows_bwd_rmsnorm(const void* dxs, const int* inv_pad, const void* addend,
                                    const void* x, const float* w, const float* rstd, long long T,
                                    int k, int H, int partial, void* dx, float* dw, void* scratch,
                                    long long scratch_bytes, void* stream) {
  REQUIRE(dxs && x && w && rstd && dx && dw && scratch, "gather_rows_bwd_rmsnorm: null pointer");
  REQUIRE(H % 8 == 0 && H > 0 && k >= 1 && k <= kMaxTopK, "gather_rows_bwd_rmsnorm: bad shape");
  REQUIRE(aligned16(dxs) && aligned16(x) && aligned16(dx) && (!addend || aligned16(addend)),
          "gather_rows_bwd_rmsnorm: 16-byte aligned rows needed");
  REQUIRE(scratch_bytes >= b200moe_gather_rows_bwd_rmsnorm_scratch_bytes(T, H),
          "gather_rows_bwd_rmsnorm: scratch too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    const cudaError_t e = cudaMemsetAsync(dw, 0, static_cast<size_t>(H) * sizeof(float), st);
    if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "gather_rows_bwd_rmsnorm: %s", cudaGetErrorString(e));
    return B200MOE_OK;
  }
  NormBwd nb;
  nb.x = static_cast<const __nv_bfloat16*>(x);
  nb.w = w;
  nb.rstd = rstd;
  nb.dw_part = static_cast<float*>(scratch);
  nb.inv_h = 1.0f / static_cast<float>(H);
  long long grid = 0;
  int rc = launch_row_reduce(static_cast<const __nv_bfloat16*>(dxs), inv_pad, nullptr,
                             static_cast<const __nv_bfloat16*>(addend), T, k, H,
                             static_cast<__nv_bfloat16*>(dx), st, "gather_rows_bwd_rmsnorm",
                             partial != 0, &nb, &grid);
  if (rc < 0)
    return fail(B200MOE_ERR_UNSUPPORTED,
                "gather_rows_bwd_rmsnorm: H*k = %lld does not fit the shared-memory row ring "
                "(H*k <= 18432, H <= 4096, H %% 32 == 0)", static_cast<long long>(H) * k);
  if (rc) return rc;
  sum_columns_kernel<<<(H + 255) / 256, 256, 0, st>>>(static_cast<const float*>(scratch),
                                                      static_cast<int>(grid * kReduceGroups), H, dw);
  return check_launch("rmsnorm_weight_grad");
}

int b200moe_combine_fwd(const void* y, const int* inv_pad, const void* weights, long long T, int k,
                        int H, int partial, void* out, void* stream) {
  REQUIRE(y && weights && out, "combine_fwd: null pointer");
  REQUIRE(H % 8 == 0 && H > 0 && k >= 1 && k <= kMaxTopK, "combine_fwd: bad shape");
  if (T == 0) return B200MOE_OK;
  {
    const int rc = launch_row_reduce(static_cast<const __nv_bfloat16*>(y), inv_pad,
                                     static_cast<const __nv_bfloat16*>(weights), nullptr, T, k, H,
                                     static_cast<__nv_bfloat16*>(out),
                                     static_cast<cudaStream_t>(stream), "combine_fwd",
                                     partial != 0);
    if (rc >= 0) return rc;
  }
  combine_fwd_kernel<<<grid_for(T, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), inv_pad, static_cast<const __nv_bfloat16*>(weights), T,
      k, H, static_cast<__nv_bfloat16*>(out));
  return check_launch("combine_fwd");
}

int b200moe_combine_bwd(const void* d_out, const void* y, const int* row_flat, const int* inv_pad,
                        const int* pad_offsets, const void* weights, int E, long long T, int k,
                        int H, long long rows_cap, int y_token_major, void* dy, float* d_weights,
                        void* stream) {
  REQUIRE(d_out && y && row_flat && pad_offsets && weights && dy && d_weights,
          "combine_bwd: null pointer");
  REQUIRE(H % 8 == 0 && H > 0 && k >= 1, "combine_bwd: bad shape");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* dyp = static_cast<__nv_bfloat16*>(dy);
  if (y_token_major) {
    REQUIRE(inv_pad, "combine_bwd: token-major y needs inv_pad");
    const long long R = T * k;
    zero_pad_rows_kernel<<<grid_for(rows_cap, 8), 256, 0, st>>>(row_flat, pad_offsets + E, H, dyp);
    int rc = check_launch("combine_bwd zero pad");
    if (rc) return rc;
    if (R == 0) return B200MOE_OK;
    combine_bwd_token_major_kernel<<<grid_for(R, 8), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(d_out), static_cast<const __nv_bfloat16*>(y), inv_pad,
        static_cast<const __nv_bfloat16*>(weights), R, k, H, dyp, d_weights);
    return check_launch("combine_bwd");
  }
  auto* dop = static_cast<const __nv_bfloat16*>(d_out);
  auto* yp = static_cast<const __nv_bfloat16*>(y);
  auto* wp = static_cast<const __nv_bfloat16*>(weights);
  if (B200MOE_TOKEN_ORDER && inv_pad && k <= 32 &&
      (H == 256 || H == 512 || H == 1024 || H == 2048)) {
    REQUIRE(T >= 0, "combine_bwd: negative T");
    const int grid = grid_for(T > rows_cap / 32 ? T : rows_cap / 32, 8);
    const int* tot = pad_offsets + E;
    switch (H) {
      case 256: combine_bwd_tokens_kernel<1><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights); break;
      case 512: combine_bwd_tokens_kernel<2><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights); break;
      case 1024: combine_bwd_tokens_kernel<4><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights); break;
      default: combine_bwd_tokens_kernel<8><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights); break;
    }
    return check_launch("combine_bwd");
  }
  if (inv_pad && T * k > 0) {  // slots without an expert have no row: their d_weights are 0
    zero_skipped_slots_kernel<<<grid_for(T * k, 256), 256, 0, st>>>(inv_pad, T * k, d_weights);
    const int rc = check_launch("combine_bwd zero skipped");
    if (rc) return rc;
  }
  const int grid = grid_for(rows_cap, 8);
  switch (H) {
    case 256: combine_bwd_kernel<1><<<grid, 256, 0, st>>>(dop, yp, row_flat, pad_offsets + E, wp, k, H, dyp, d_weights); break;
    case 512: combine_bwd_kernel<2><<<grid, 256, 0, st>>>(dop, yp, row_flat, pad_offsets + E, wp, k, H, dyp, d_weights); break;
    case 1024: combine_bwd_kernel<4><<<grid, 256, 0, st>>>(dop, yp, row_flat, pad_offsets + E, wp, k, H, dyp, d_weights); break;
    case 2048: combine_bwd_kernel<8><<<grid, 256, 0, st>>>(dop, yp, row_flat, pad_offsets + E, wp, k, H, dyp, d_weights); break;
    default: combine_bwd_kernel<0><<<grid, 256, 0, st>>>(dop, yp, row_flat, pad_offsets + E, wp, k, H, dyp, d_weights); break;
  }
  return check_launch("combine_bwd");
}

// ---------------------------------------------------------------- expert GEMMs
static int check_expert_shape(const char* what, long long rows_cap, int E, int H, int I) {
  REQUIRE(E >= 1 && E <= 4096, "%s: bad E", what);
  REQUIRE(H > 0 && H % 128 == 0, "%s: H must be a multiple of 128", what);
  REQUIRE(I > 0 && I % 64 == 0, "%s: I must be a multiple of 64", what);
  REQUIRE(rows_cap > 0 && rows_cap % 128 == 0 && rows_cap < 0x7fffffffLL,
          "%s: rows_cap must be a positive multiple of 128", what);
  REQUIRE(static_cast<long long>(E) * 2 * I < 0x7fffffffLL && static_cast<long long>(E) * H < 0x7fffffffLL,
          "%s: weights too large", what);
  return B200MOE_OK;
}

int b200moe_expert_gate_up_fwd(const void* xs, const void* w_gu, const int* tile_expert,
                               const int* pad_offsets, long long rows_cap, int E, int H, int I,
                               void* gu, void* h, void* stream) {
  REQUIRE(xs && w_gu && tile_expert && pad_offsets && gu && h, "gate_up_fwd: null pointer");
  int rc = check_expert_shape("gate_up_fwd", rows_cap, E, H, I);
  if (rc) return rc;
  const int half = (I % 128 == 0) ? 128 : 64;  // BN = 2*half: gate and up halves
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, xs, H, rows_cap, H, 64, 128, "gate_up_fwd xs"))) return rc;
  if ((rc = make_tmap(&tb, w_gu, H, static_cast<long long>(E) * 2 * I, H, 64, half,
                      "gate_up_fwd w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = I / half;
  p.k_blocks = H / 64;
  p.b_group_rows = 2 * I;
  p.b_half_offset = I;
  p.m_valid = rows_cap;
  p.n_valid = I;
  p.out = gu;
  p.ld_out = 2 * I;
  p.out2 = h;
  p.ld_out2 = I;
  p.inter = I;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap to0, to1;
  if ((rc = make_out_tmap(&to0, gu, 2LL * I, rows_cap, "gate_up_fwd gu"))) return rc;
  if ((rc = make_out_tmap(&to1, h, I, rows_cap, "gate_up_fwd h"))) return rc;
  if (half == 128)
    return launch_expert_gemm<256, false, false, kEpiSwigluFwd, kRowsRagged>(ta, tb, p, st, "gate_up_fwd", &to0, &to1);
  return launch_expert_gemm<128, false, false, kEpiSwigluFwd, kRowsRagged>(ta, tb, p, st, "gate_up_fwd", &to0, &to1);
}

int b200moe_expert_down_fwd(const void* h, const void* w_d, const int* tile_expert,
                            const int* pad_offsets, const int* row_flat_out, long long rows_cap,
                            int E, int H, int I, void* y, void* stream) {
  REQUIRE(h && w_d && tile_expert && pad_offsets && y, "down_fwd: null pointer");
  int rc = check_expert_shape("down_fwd", rows_cap, E, H, I);
  if (rc) return rc;
  const int BN = (H % 256 == 0) ? 256 : 128;
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, h, I, rows_cap, I, 64, 128, "down_fwd h"))) return rc;
  const int b_box = use_pair(BN, kRowsRagged, E, 0) ? BN / 2 : BN;
  if ((rc = make_tmap(&tb, w_d, I, static_cast<long long>(E) * H, I, 64, b_box, "down_fwd w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = H / BN;
  p.k_blocks = I / 64;
  p.b_group_rows = H;
  p.m_valid = rows_cap;
  p.n_valid = H;
  p.out = y;
  p.ld_out = H;
  p.scatter_rows = row_flat_out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap to0;
  const CUtensorMap* o0 = nullptr;
  if (row_flat_out == nullptr) {
    if ((rc = make_store_tmap(&to0, y, H, rows_cap, "down_fwd y"))) return rc;
    o0 = &to0;
  }
  if (BN == 256) return launch_expert_gemm<256, false, false, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "down_fwd", o0);
  return launch_expert_gemm<128, false, false, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "down_fwd", o0);
}

int b200moe_expert_down_dgrad_swiglu(const void* dy, const void* w_d, const void* gu,
                                     const int* tile_expert, const int* pad_offsets,
                                     long long rows_cap, int E, int H, int I, void* d_gu,
                                     void* stream) {
  REQUIRE(dy && w_d && gu && tile_expert && pad_offsets && d_gu, "down_dgrad: null pointer");
  int rc = check_expert_shape("down_dgrad", rows_cap, E, H, I);
  if (rc) return rc;
  const int BN = (I % 256 == 0) ? 256 : (I % 128 == 0 ? 128 : 64);
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, dy, H, rows_cap, H, 64, 128, "down_dgrad dy"))) return rc;
  // B[n=i][k=h] = W_d[e][h][i]: MN-major, rows (e*H + h), columns i
  if ((rc = make_tmap(&tb, w_d, I, static_cast<long long>(E) * H, I, 64, 64, "down_dgrad w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = I / BN;
  p.k_blocks = H / 64;
  p.b_group_rows = H;
  p.m_valid = rows_cap;
  p.n_valid = I;
  p.out = d_gu;
  p.ld_out = 2 * I;
  p.aux = gu;
  p.ld_aux = 2 * I;
  p.inter = I;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap to0, to1;  // d_gu out, gu in (the pair kernel's epilogue loads it by TMA)
  if ((rc = make_out_tmap(&to0, d_gu, 2LL * I, rows_cap, "down_dgrad d_gu"))) return rc;
  if ((rc = make_out_tmap(&to1, gu, 2LL * I, rows_cap, "down_dgrad gu"))) return rc;
  if (BN == 256) return launch_expert_gemm<256, false, true, kEpiSwigluBwd, kRowsRagged>(ta, tb, p, st, "down_dgrad", &to0, &to1);
  if (BN == 128) return launch_expert_gemm<128, false, true, kEpiSwigluBwd, kRowsRagged>(ta, tb, p, st, "down_dgrad", &to0, &to1);
  return launch_expert_gemm<64, false, true, kEpiSwigluBwd, kRowsRagged>(ta, tb, p, st, "down_dgrad");
}

int b200moe_expert_gate_up_dgrad(const void* d_gu, const void* w_gu, const int* tile_expert,
                                 const int* pad_offsets, const int* row_flat_out,
                                 long long rows_cap, int E, int H, int I, void* dxs, void* stream) {
  REQUIRE(d_gu && w_gu && tile_expert && pad_offsets && dxs, "gate_up_dgrad: null pointer");
  int rc = check_expert_shape("gate_up_dgrad", rows_cap, E, H, I);
  if (rc) return rc;
  const int BN = (H % 256 == 0) ? 256 : 128;
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, d_gu, 2 * I, rows_cap, 2 * I, 64, 128, "gate_up_dgrad d_gu"))) return rc;
  // B[n=h][k=j] = W_gu[e][j][h]: MN-major, rows (e*2I + j), columns h
  if ((rc = make_tmap(&tb, w_gu, H, static_cast<long long>(E) * 2 * I, H, 64, 64,
                      "gate_up_dgrad w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = H / BN;
  p.k_blocks = 2 * I / 64;
  p.b_group_rows = 2 * I;
  p.m_valid = rows_cap;
  p.n_valid = H;
  p.out = dxs;
  p.ld_out = H;
  p.scatter_rows = row_flat_out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap to0;
  const CUtensorMap* o0 = nullptr;
  if (row_flat_out == nullptr) {
    if ((rc = make_store_tmap(&to0, dxs, H, rows_cap, "gate_up_dgrad dxs"))) return rc;
    o0 = &to0;
  }
  if (BN == 256) return launch_expert_gemm<256, false, true, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "gate_up_dgrad", o0);
  return launch_expert_gemm<128, false, true, kEpiStoreBf16, kRowsRagged>(ta, tb, p, st, "gate_up_dgrad", o0);
}

int b200moe_expert_wgrad(const void* a, int M, const void* b, int N, const int* pad_offsets, int E,
                         long long rows_cap, float* dw, int accumulate, void* stream) {
  REQUIRE(a && b && pad_offsets && dw, "expert_wgrad: null pointer");
  REQUIRE(M > 0 && M % 128 == 0, "expert_wgrad: M must be a multiple of 128");
  REQUIRE(N > 0 && N % 64 == 0, "expert_wgrad: N must be a multiple of 64");
  REQUIRE(E >= 1 && rows_cap > 0 && rows_cap % 128 == 0, "expert_wgrad: bad rows/E");
  const int BN = (N % 256 == 0) ? 256 : (N % 128 == 0 ? 128 : 64);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, a, M, rows_cap, M, 64, 64, "expert_wgrad a"))) return rc;
  if ((rc = make_tmap(&tb, b, N, rows_cap, N, 64, 64, "expert_wgrad b"))) return rc;
  GemmParams p = blank_params();
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.m_tiles = M / 128;
  p.n_tiles = N / BN;
  p.n_valid = N;
  p.out = dw;
  p.ld_out = N;
  p.accumulate = accumulate;
  p.out_group_stride = static_cast<long long>(M) * N;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN >= 128 && use_pair(BN, kKRagged, E, p.m_tiles)) {
    // two-CTA tiles whose fp32 output leaves through shared memory with TMA
    // stores (reduce-adds when accumulating): coalesced and asynchronous
    CUtensorMap to;
    if ((rc = make_wgrad_tmap(&to, dw, N, static_cast<long long>(E) * M, "expert_wgrad dw")))
      return rc;
    if (BN == 256)
      return launch_gemm_pair<256, true, true, kEpiStoreF32Tma, kKRagged>(ta, tb, to, to, p, st,
                                                                          "expert_wgrad");
    return launch_gemm_pair<128, true, true, kEpiStoreF32Tma, kKRagged>(ta, tb, to, to, p, st,
                                                                        "expert_wgrad");
  }
  if (BN == 256) return launch_expert_gemm<256, true, true, kEpiStoreF32, kKRagged>(ta, tb, p, st, "expert_wgrad");
  if (BN == 128) return launch_expert_gemm<128, true, true, kEpiStoreF32, kKRagged>(ta, tb, p, st, "expert_wgrad");
  return launch_expert_gemm<64, true, true, kEpiStoreF32, kKRagged>(ta, tb, p, st, "expert_wgrad");
}

int b200moe_expert_wgrad_segments(const void* a, int M, const void* b, int N,
                                  const int* seg_offsets, int segments, int E,
                                  long long rows_total, float* dw, int accumulate, void* stream) {
  REQUIRE(a && b && seg_offsets && dw, "expert_wgrad_segments: null pointer");
  REQUIRE(M > 0 && M % 128 == 0, "expert_wgrad_segments: M must be a multiple of 128");
  REQUIRE(N > 0 && N % 64 == 0, "expert_wgrad_segments: N must be a multiple of 64");
  REQUIRE(E >= 1 && rows_total > 0 && rows_total % 128 == 0 && rows_total < 0x7fffffffLL,
          "expert_wgrad_segments: bad rows/E");
  REQUIRE(segments >= 1 && segments <= kMaxWgradSegments,
          "expert_wgrad_segments: 1 <= segments <= %d", kMaxWgradSegments);
  const int BN = N % 256 == 0 ? 256 : 128;
  if (N < 128 || !use_pair(BN, kKRagged, E, M / 128)) {
    // shapes the two-CTA tiles do not take: one weight gradient per segment,
    // each after the first added into dw
    for (int s = 0; s < segments; ++s) {
      const int rc = b200moe_expert_wgrad(a, M, b, N, seg_offsets + static_cast<long long>(s) * (E + 1),
                                          E, rows_total, dw, accumulate || s > 0, stream);
      if (rc) return rc;
    }
    return B200MOE_OK;
  }
  CUtensorMap ta, tb, to;
  int rc;
  if ((rc = make_tmap(&ta, a, M, rows_total, M, 64, 64, "expert_wgrad_segments a"))) return rc;
  if ((rc = make_tmap(&tb, b, N, rows_total, N, 64, 64, "expert_wgrad_segments b"))) return rc;
  if ((rc = make_wgrad_tmap(&to, dw, N, static_cast<long long>(E) * M,
                              "expert_wgrad_segments dw")))
    return rc;
  GemmParams p = blank_params();
  p.pad_offsets = seg_offsets;
  p.k_segments = segments;
  p.num_groups = E;
  p.m_tiles = M / 128;
  p.n_tiles = (N + BN - 1) / BN;  // columns past N: zero-filled loads, not stored
  p.n_valid = N;
  p.out = dw;
  p.ld_out = N;
  p.accumulate = accumulate;
  p.out_group_stride = static_cast<long long>(M) * N;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 256)
    return launch_gemm_pair<256, true, true, kEpiStoreF32Tma, kKRagged>(ta, tb, to, to, p, st,
                                                                        "expert_wgrad_segments");
  return launch_gemm_pair<128, true, true, kEpiStoreF32Tma, kKRagged>(ta, tb, to, to, p, st,
                                                                      "expert_wgrad_segments");
}

// ---------------------------------------------------------------- fp8 expert path
// spark-gpt's --fp8-mlp on MoE layers (train.py:1301-1604): e4m3 x, gu, h and
// weights, e5m2 d_gu and dy, delayed per-site scales (scale[0..4] = x, gu, h,
// d_gu, dy) read from device memory, amax slots raised by the kernels that
// quantize.  Every GEMM is a two-CTA pair kernel; shapes as the reference's
// gate (H a multiple of 256 here, I of 128, E <= 256).
static int check_fp8_shape(const char* what, long long rows_cap, int E, int H, int I) {
  REQUIRE(E >= 1 && E <= kMaxPairExperts, "%s: fp8 expert GEMMs take 1 <= E <= %d", what,
          kMaxPairExperts);
  REQUIRE(H > 0 && H % 256 == 0, "%s: fp8 path needs H a multiple of 256", what);
  REQUIRE(I > 0 && I % 128 == 0, "%s: fp8 path needs I a multiple of 128", what);
  REQUIRE(rows_cap > 0 && rows_cap % 128 == 0 && rows_cap < 0x7fffffffLL,
          "%s: rows_cap must be a positive multiple of 128", what);
  REQUIRE(static_cast<long long>(E) * 2 * I < 0x7fffffffLL && static_cast<long long>(E) * H < 0x7fffffffLL,
          "%s: weights too large", what);
  REQUIRE(g_pair_gemm, "%s: the fp8 path runs only as two-CTA pair tiles", what);
  return B200MOE_OK;
}

long long b200moe_fp8_quantize_experts_scratch_bytes(int E) {
  return static_cast<long long>(E > 0 ? E : 1) * 64 * static_cast<long long>(sizeof(float));
}

int b200moe_fp8_quantize_experts(const float* w, int E, long long per_expert, void* w8, float* q,
                                 void* scratch, long long scratch_bytes, void* stream) {
  REQUIRE(w && w8 && q && scratch, "fp8_quantize_experts: null pointer");
  REQUIRE(E >= 1 && E <= 65535 && per_expert > 0 && per_expert % 4 == 0,
          "fp8_quantize_experts: need 1 <= E <= 65535 and a per-expert size that is a "
          "multiple of 4");
  REQUIRE(aligned16(w) && aligned16(w8), "fp8_quantize_experts: pointers must be 16-byte aligned");
  REQUIRE(scratch_bytes >= b200moe_fp8_quantize_experts_scratch_bytes(E),
          "fp8_quantize_experts: scratch too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // splits per expert: about four blocks per SM over all experts, at most 64
  int splits = static_cast<int>((4LL * num_sms() + E - 1) / E);
  splits = std::max(1, std::min(64, splits));
  float* partial = static_cast<float*>(scratch);
  fp8_weight_amax_kernel<<<dim3(splits, E), kWeightAmaxThreads, 0, st>>>(w, per_expert, splits,
                                                                          partial);
  int rc = check_launch("fp8_quantize_experts amax");
  if (rc) return rc;
  fp8_weight_scale_kernel<<<(E + 127) / 128, 128, 0, st>>>(partial, E, splits, q);
  if ((rc = check_launch("fp8_quantize_experts scale"))) return rc;
  const long long total = static_cast<long long>(E) * per_expert;
  fp8_weight_quant_kernel<<<grid_for(total / 4, 256), 256, 0, st>>>(w, per_expert, total, q,
                                                                    static_cast<uint8_t*>(w8));
  return check_launch("fp8_quantize_experts quant");
}

int b200moe_fp8_gather_quant(const void* x, const int* row_flat, const int* inv_pad,
                             const int* pad_offsets, long long T, int E, int k, int H,
                             long long rows_cap, const float* scale, float* amax, void* x8,
                             void* stream) {
  REQUIRE(x && row_flat && inv_pad && pad_offsets && scale && amax && x8,
          "fp8_gather_quant: null pointer");
  REQUIRE(H > 0 && H % 16 == 0 && k >= 1 && k <= 32 && T >= 0,
          "fp8_gather_quant: need H a multiple of 16 and 1 <= k <= 32");
  REQUIRE(aligned16(x) && aligned16(x8), "fp8_gather_quant: pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(T > rows_cap / 32 ? T : rows_cap / 32, 8);
  fp8_gather_quant_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), inv_pad,
                                                row_flat, pad_offsets + E, T, k, H, scale, amax,
                                                static_cast<uint8_t*>(x8));
  return check_launch("fp8_gather_quant");
}

int b200moe_fp8_quantize_rows(const void* src, long long rows, int cols, const int* total_rows,
                              const float* scale, float* amax, int fmt, void* dst, void* stream) {
  REQUIRE(src && scale && amax && dst, "fp8_quantize_rows: null pointer");
  REQUIRE(rows >= 0 && cols > 0 && cols % 8 == 0, "fp8_quantize_rows: cols must be a multiple of 8");
  REQUIRE(fmt == 0 || fmt == 1, "fp8_quantize_rows: fmt 0 (e4m3) or 1 (e5m2)");
  REQUIRE(aligned16(src) && aligned16(dst), "fp8_quantize_rows: pointers must be 16-byte aligned");
  const long long n8 = rows * cols / 8;
  if (n8 == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(n8, 256);
  if (fmt == 0)
    fp8_quantize_rows_kernel<kE4M3><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(src), n8, cols, total_rows, scale, amax,
        static_cast<uint8_t*>(dst));
  else
    fp8_quantize_rows_kernel<kE5M2><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(src), n8, cols, total_rows, scale, amax,
        static_cast<uint8_t*>(dst));
  return check_launch("fp8_quantize_rows");
}

int b200moe_fp8_combine_bwd(const void* d_out, const void* y, const int* row_flat,
                            const int* inv_pad, const int* pad_offsets, const void* weights,
                            int E, long long T, int k, int H, long long rows_cap,
                            const float* scale_dy, float* amax_dy, void* dy, float* d_weights,
                            void* dy8, void* stream) {
  REQUIRE(d_out && y && row_flat && inv_pad && pad_offsets && weights && dy && d_weights &&
              scale_dy && amax_dy && dy8,
          "fp8_combine_bwd: null pointer");
  REQUIRE(H % 16 == 0 && H > 0 && k >= 1 && T >= 0, "fp8_combine_bwd: bad shape");
  REQUIRE(aligned16(dy) && aligned16(dy8), "fp8_combine_bwd: pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!(B200MOE_TOKEN_ORDER && k <= 32 && (H == 256 || H == 512 || H == 1024 || H == 2048))) {
    // other shapes: the plain combine backward, then the e5m2 copy of its rows
    int rc = b200moe_combine_bwd(d_out, y, row_flat, inv_pad, pad_offsets, weights, E, T, k, H,
                                 rows_cap, 0, dy, d_weights, stream);
    if (rc) return rc;
    return b200moe_fp8_quantize_rows(dy, rows_cap, H, pad_offsets + E, scale_dy, amax_dy, 1, dy8,
                                     stream);
  }
  auto* dop = static_cast<const __nv_bfloat16*>(d_out);
  auto* yp = static_cast<const __nv_bfloat16*>(y);
  auto* wp = static_cast<const __nv_bfloat16*>(weights);
  auto* dyp = static_cast<__nv_bfloat16*>(dy);
  auto* d8 = static_cast<uint8_t*>(dy8);
  const int grid = grid_for(T > rows_cap / 32 ? T : rows_cap / 32, 8);
  const int* tot = pad_offsets + E;
  switch (H) {
    case 256: combine_bwd_tokens_kernel<1, true><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights, scale_dy, amax_dy, d8); break;
    case 512: combine_bwd_tokens_kernel<2, true><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights, scale_dy, amax_dy, d8); break;
    case 1024: combine_bwd_tokens_kernel<4, true><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights, scale_dy, amax_dy, d8); break;
    default: combine_bwd_tokens_kernel<8, true><<<grid, 256, 0, st>>>(dop, yp, inv_pad, row_flat, tot, wp, T, k, H, dyp, d_weights, scale_dy, amax_dy, d8); break;
  }
  return check_launch("fp8_combine_bwd");
}

int b200moe_fp8_expert_gate_up_fwd(const void* x8, const void* w8_gu, const float* q_gu,
                                   const int* tile_expert, const int* pad_offsets,
                                   long long rows_cap, int E, int H, int I, const float* scale,
                                   float* amax, void* gu8, void* h8, void* stream) {
  REQUIRE(x8 && w8_gu && q_gu && tile_expert && pad_offsets && scale && amax && gu8 && h8,
          "fp8_gate_up_fwd: null pointer");
  int rc = check_fp8_shape("fp8_gate_up_fwd", rows_cap, E, H, I);
  if (rc) return rc;
  CUtensorMap ta, tb;
  if ((rc = make_tmap_u8(&ta, x8, H, rows_cap, H, 128, 128, "fp8_gate_up_fwd x8"))) return rc;
  if ((rc = make_tmap_u8(&tb, w8_gu, H, static_cast<long long>(E) * 2 * I, H, 128, 128,
                         "fp8_gate_up_fwd w8")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = I / 128;
  p.k_blocks = H / 128;
  p.b_group_rows = 2 * I;
  p.b_half_offset = I;
  p.m_valid = rows_cap;
  p.n_valid = I;
  p.out = gu8;
  p.ld_out = 2 * I;
  p.out2 = h8;
  p.ld_out2 = I;
  p.inter = I;
  p.fp8_scale = scale;
  p.fp8_amax = amax;
  p.deq_a = scale;  // x
  p.deq_g = q_gu;
  CUtensorMap to0, to1;
  if ((rc = make_out_tmap_u8(&to0, gu8, 2LL * I, rows_cap, "fp8_gate_up_fwd gu8"))) return rc;
  if ((rc = make_out_tmap_u8(&to1, h8, I, rows_cap, "fp8_gate_up_fwd h8"))) return rc;
  return launch_gemm_pair<256, false, false, kEpiSwigluFwdF8, kRowsRagged, kOpE4m3>(
      ta, tb, to0, to1, p, static_cast<cudaStream_t>(stream), "fp8_gate_up_fwd");
}

int b200moe_fp8_expert_down_fwd(const void* h8, const void* wd8, const float* q_d,
                                const int* tile_expert, const int* pad_offsets, long long rows_cap,
                                int E, int H, int I, const float* scale, void* y, void* stream) {
  REQUIRE(h8 && wd8 && q_d && tile_expert && pad_offsets && scale && y, "fp8_down_fwd: null pointer");
  int rc = check_fp8_shape("fp8_down_fwd", rows_cap, E, H, I);
  if (rc) return rc;
  CUtensorMap ta, tb, to0;
  if ((rc = make_tmap_u8(&ta, h8, I, rows_cap, I, 128, 128, "fp8_down_fwd h8"))) return rc;
  if ((rc = make_tmap_u8(&tb, wd8, I, static_cast<long long>(E) * H, I, 128, 128, "fp8_down_fwd w8")))
    return rc;
  if ((rc = make_store_tmap(&to0, y, H, rows_cap, "fp8_down_fwd y"))) return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = H / 256;
  p.k_blocks = I / 128;
  p.b_group_rows = H;
  p.m_valid = rows_cap;
  p.n_valid = H;
  p.out = y;
  p.ld_out = H;
  p.deq_a = scale + 2;  // h
  p.deq_g = q_d;
  return launch_gemm_pair<256, false, false, kEpiStoreBf16, kRowsRagged, kOpE4m3>(
      ta, tb, to0, to0, p, static_cast<cudaStream_t>(stream), "fp8_down_fwd");
}

int b200moe_fp8_expert_down_dgrad_swiglu(const void* dy, const void* w_d, const void* gu8,
                                         const int* tile_expert, const int* pad_offsets,
                                         long long rows_cap, int E, int H, int I,
                                         const float* scale, float* amax, void* d_gu8,
                                         void* stream) {
  REQUIRE(dy && w_d && gu8 && tile_expert && pad_offsets && scale && amax && d_gu8,
          "fp8_down_dgrad: null pointer");
  int rc = check_fp8_shape("fp8_down_dgrad", rows_cap, E, H, I);
  if (rc) return rc;
  REQUIRE(aligned16(gu8) && aligned16(d_gu8), "fp8_down_dgrad: pointers must be 16-byte aligned");
  const int BN = (I % 256 == 0) ? 256 : 128;
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, dy, H, rows_cap, H, 64, 128, "fp8_down_dgrad dy"))) return rc;
  if ((rc = make_tmap(&tb, w_d, I, static_cast<long long>(E) * H, I, 64, 64, "fp8_down_dgrad w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = I / BN;
  p.k_blocks = H / 64;
  p.b_group_rows = H;
  p.m_valid = rows_cap;
  p.n_valid = I;
  p.out = d_gu8;
  p.ld_out = 2 * I;
  p.aux = gu8;
  p.ld_aux = 2 * I;
  p.inter = I;
  p.fp8_scale = scale;
  p.fp8_amax = amax;
  CUtensorMap to0, to1;  // d_gu8 out, gu8 in (loaded by TMA in the epilogue)
  if ((rc = make_out_tmap_u8(&to0, d_gu8, 2LL * I, rows_cap, "fp8_down_dgrad d_gu8"))) return rc;
  if ((rc = make_out_tmap_u8(&to1, gu8, 2LL * I, rows_cap, "fp8_down_dgrad gu8"))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 256)
    return launch_gemm_pair<256, false, true, kEpiSwigluBwdF8, kRowsRagged>(ta, tb, to0, to1, p,
                                                                            st, "fp8_down_dgrad");
  return launch_gemm_pair<128, false, true, kEpiSwigluBwdF8, kRowsRagged>(ta, tb, to0, to1, p, st,
                                                                          "fp8_down_dgrad");
}

int b200moe_fp8_expert_gate_up_dgrad(const void* d_gu8, const void* w8_gu, const float* q_gu,
                                     const int* tile_expert, const int* pad_offsets,
                                     long long rows_cap, int E, int H, int I, const float* scale,
                                     void* dxs, void* stream) {
  REQUIRE(d_gu8 && w8_gu && q_gu && tile_expert && pad_offsets && scale && dxs,
          "fp8_gate_up_dgrad: null pointer");
  int rc = check_fp8_shape("fp8_gate_up_dgrad", rows_cap, E, H, I);
  if (rc) return rc;
  CUtensorMap ta, tb, to0;
  if ((rc = make_tmap_u8(&ta, d_gu8, 2 * I, rows_cap, 2 * I, 128, 128, "fp8_gate_up_dgrad d_gu8")))
    return rc;
  // B[n=h][k=j] = W8_gu[e][j][h]: MN-major, rows (e*2I + j), columns h
  if ((rc = make_tmap_u8(&tb, w8_gu, H, static_cast<long long>(E) * 2 * I, H, 128, 128,
                         "fp8_gate_up_dgrad w8")))
    return rc;
  if ((rc = make_store_tmap(&to0, dxs, H, rows_cap, "fp8_gate_up_dgrad dxs"))) return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = H / 256;
  p.k_blocks = 2 * I / 128;
  p.b_group_rows = 2 * I;
  p.m_valid = rows_cap;
  p.n_valid = H;
  p.out = dxs;
  p.ld_out = H;
  p.deq_a = scale + 3;  // d_gu
  p.deq_g = q_gu;
  return launch_gemm_pair<256, false, true, kEpiStoreBf16, kRowsRagged, kOpE5m2E4m3>(
      ta, tb, to0, to0, p, static_cast<cudaStream_t>(stream), "fp8_gate_up_dgrad");
}

int b200moe_fp8_expert_wgrad(const void* a8, int a_fmt, int M, const void* b8, int N,
                             const int* pad_offsets, int E, long long rows_cap,
                             const float* scale_a, const float* scale_b, float* dw, int accumulate,
                             void* stream) {
  REQUIRE(a8 && b8 && pad_offsets && scale_a && scale_b && dw, "fp8_wgrad: null pointer");
  REQUIRE(a_fmt == 0 || a_fmt == 1, "fp8_wgrad: a_fmt 0 (e4m3) or 1 (e5m2)");
  REQUIRE(M > 0 && M % 256 == 0, "fp8_wgrad: M must be a multiple of 256");
  REQUIRE(N > 0 && N % 128 == 0, "fp8_wgrad: N must be a multiple of 128");
  REQUIRE(E >= 1 && E <= kMaxPairExperts && rows_cap > 0 && rows_cap % 128 == 0,
          "fp8_wgrad: bad rows/E");
  REQUIRE(g_pair_gemm, "fp8_wgrad: the fp8 path runs only as two-CTA pair tiles");
  CUtensorMap ta, tb, to;
  int rc;
  if ((rc = make_tmap_u8(&ta, a8, M, rows_cap, M, 128, 128, "fp8_wgrad a"))) return rc;
  if ((rc = make_tmap_u8(&tb, b8, N, rows_cap, N, 128, 128, "fp8_wgrad b"))) return rc;
  if ((rc = make_wgrad_tmap(&to, dw, N, static_cast<long long>(E) * M, "fp8_wgrad dw"))) return rc;
  GemmParams p = blank_params();
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.m_tiles = M / 128;
  p.n_tiles = (N + 255) / 256;  // a last half tile reads zero columns; its stores are clipped
  p.n_valid = N;
  p.out = dw;
  p.ld_out = N;
  p.accumulate = accumulate;
  p.out_group_stride = static_cast<long long>(M) * N;
  p.deq_a = scale_a;
  p.deq_b = scale_b;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a_fmt == 1)
    return launch_gemm_pair<256, true, true, kEpiStoreF32Tma, kKRagged, kOpE5m2E4m3>(
        ta, tb, to, to, p, st, "fp8_wgrad");
  return launch_gemm_pair<256, true, true, kEpiStoreF32Tma, kKRagged, kOpE4m3>(ta, tb, to, to, p,
                                                                             st, "fp8_wgrad");
}

// ---------------------------------------------------------------- gathered-operand GEMMs
int b200moe_expert_gate_up_fwd_gather(const void* x, const int* row_flat, long long T, int k,
                                      const void* w_gu, const int* tile_expert,
                                      const int* pad_offsets, long long rows_cap, int E, int H,
                                      int I, void* gu, void* h, void* stream) {
  REQUIRE(x && row_flat && w_gu && tile_expert && pad_offsets && gu && h,
          "gate_up_fwd_gather: null pointer");
  int rc = check_expert_shape("gate_up_fwd_gather", rows_cap, E, H, I);
  if (rc) return rc;
  REQUIRE(T > 0 && T < 0x7fffffffLL && k >= 1, "gate_up_fwd_gather: bad T/k");
  const int half = (I % 128 == 0) ? 128 : 64;
  CUtensorMap ta, tb;
  if ((rc = make_gather_tmap(&ta, x, H, T, "gate_up_fwd_gather x"))) return rc;
  if ((rc = make_tmap(&tb, w_gu, H, static_cast<long long>(E) * 2 * I, H, 64, half,
                      "gate_up_fwd_gather w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = I / half;
  p.k_blocks = H / 64;
  p.b_group_rows = 2 * I;
  p.b_half_offset = I;
  p.m_valid = rows_cap;
  p.n_valid = I;
  p.out = gu;
  p.ld_out = 2 * I;
  p.out2 = h;
  p.ld_out2 = I;
  p.inter = I;
  p.gather_rows = row_flat;
  p.gather_k = k;
  p.gather_oob = static_cast<int>(T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (half == 128)
    return launch_gemm<256, false, false, kEpiSwigluFwd, kRowsRagged, kGatherA>(ta, tb, p, st,
                                                                              "gate_up_fwd_gather");
  return launch_gemm<128, false, false, kEpiSwigluFwd, kRowsRagged, kGatherA>(ta, tb, p, st,
                                                                            "gate_up_fwd_gather");
}

static int down_dgrad_bn(int I) { return (I % 256 == 0) ? 256 : (I % 128 == 0 ? 128 : 64); }

long long b200moe_down_dgrad_combine_scratch_bytes(long long rows_cap, int I) {
  if (I <= 0 || I % 64) return 0;
  return 2LL * (I / down_dgrad_bn(I)) * rows_cap * static_cast<long long>(sizeof(float));
}

int b200moe_expert_down_dgrad_combine(const void* d_out, const int* row_flat, const void* weights,
                                      long long T, int k, const void* w_d, const void* gu,
                                      const void* h, const int* tile_expert,
                                      const int* pad_offsets, long long rows_cap, int E, int H,
                                      int I, void* d_gu, void* hw, float* d_weights,
                                      void* scratch, long long scratch_bytes, void* stream) {
  REQUIRE(d_out && row_flat && weights && w_d && gu && h && tile_expert && pad_offsets && d_gu &&
              hw && d_weights && scratch,
          "down_dgrad_combine: null pointer");
  int rc = check_expert_shape("down_dgrad_combine", rows_cap, E, H, I);
  if (rc) return rc;
  REQUIRE(T > 0 && T < 0x7fffffffLL && k >= 1, "down_dgrad_combine: bad T/k");
  REQUIRE(scratch_bytes >= b200moe_down_dgrad_combine_scratch_bytes(rows_cap, I),
          "down_dgrad_combine: scratch too small");
  const int BN = down_dgrad_bn(I);
  CUtensorMap ta, tb;
  if ((rc = make_gather_tmap(&ta, d_out, H, T, "down_dgrad_combine d_out"))) return rc;
  if ((rc = make_tmap(&tb, w_d, I, static_cast<long long>(E) * H, I, 64, 64,
                      "down_dgrad_combine w")))
    return rc;
  GemmParams p = blank_params();
  p.tile_expert = tile_expert;
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.n_tiles = I / BN;
  p.k_blocks = H / 64;
  p.b_group_rows = H;
  p.m_valid = rows_cap;
  p.n_valid = I;
  p.out = d_gu;
  p.ld_out = 2 * I;
  p.out2 = hw;
  p.ld_out2 = I;
  p.aux = gu;
  p.ld_aux = 2 * I;
  p.aux2 = h;
  p.ld_aux2 = I;
  p.inter = I;
  p.gather_rows = row_flat;
  p.gather_k = k;
  p.gather_oob = static_cast<int>(T);
  p.route_w = static_cast<const __nv_bfloat16*>(weights);
  p.dw_part = static_cast<float*>(scratch);
  p.part_stride = rows_cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 256)
    rc = launch_gemm<256, false, true, kEpiSwigluBwdCombine, kRowsRagged, kGatherA>(ta, tb, p, st, "down_dgrad_combine");
  else if (BN == 128)
    rc = launch_gemm<128, false, true, kEpiSwigluBwdCombine, kRowsRagged, kGatherA>(ta, tb, p, st, "down_dgrad_combine");
  else
    rc = launch_gemm<64, false, true, kEpiSwigluBwdCombine, kRowsRagged, kGatherA>(ta, tb, p, st, "down_dgrad_combine");
  if (rc) return rc;
  combine_weight_grad_kernel<<<grid_for(rows_cap, 256), 256, 0, st>>>(
      static_cast<const float*>(scratch), 2 * (I / BN), rows_cap, row_flat, pad_offsets + E,
      d_weights);
  return check_launch("combine_weight_grad");
}

static int wgrad_bn(int N) { return (N % 256 == 0) ? 256 : (N % 128 == 0 ? 128 : 64); }

int b200moe_expert_wgrad_gather_b(const void* a, int M, const void* x, int N, const int* row_flat,
                                  long long T, int k, const int* pad_offsets, int E,
                                  long long rows_cap, float* dw, int accumulate, void* stream) {
  REQUIRE(a && x && row_flat && pad_offsets && dw, "wgrad_gather_b: null pointer");
  REQUIRE(M > 0 && M % 128 == 0, "wgrad_gather_b: M must be a multiple of 128");
  REQUIRE(N > 0 && N % 64 == 0, "wgrad_gather_b: N must be a multiple of 64");
  REQUIRE(E >= 1 && rows_cap > 0 && rows_cap % 128 == 0, "wgrad_gather_b: bad rows/E");
  REQUIRE(T > 0 && T < 0x7fffffffLL && k >= 1, "wgrad_gather_b: bad T/k");
  const int BN = wgrad_bn(N);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, a, M, rows_cap, M, 64, 64, "wgrad_gather_b a"))) return rc;
  if ((rc = make_gather_tmap(&tb, x, N, T, "wgrad_gather_b x"))) return rc;
  GemmParams p = blank_params();
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.m_tiles = M / 128;
  p.n_tiles = N / BN;
  p.n_valid = N;
  p.out = dw;
  p.ld_out = N;
  p.accumulate = accumulate;
  p.out_group_stride = static_cast<long long>(M) * N;
  p.gather_rows = row_flat;
  p.gather_k = k;
  p.gather_oob = static_cast<int>(T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 256) return launch_gemm<256, true, true, kEpiStoreF32, kKRagged, kGatherB>(ta, tb, p, st, "wgrad_gather_b");
  if (BN == 128) return launch_gemm<128, true, true, kEpiStoreF32, kKRagged, kGatherB>(ta, tb, p, st, "wgrad_gather_b");
  return launch_gemm<64, true, true, kEpiStoreF32, kKRagged, kGatherB>(ta, tb, p, st, "wgrad_gather_b");
}

int b200moe_expert_wgrad_gather_a(const void* src, int M, const int* row_flat, long long T, int k,
                                  const void* b, int N, const int* pad_offsets, int E,
                                  long long rows_cap, float* dw, int accumulate, void* stream) {
  REQUIRE(src && row_flat && b && pad_offsets && dw, "wgrad_gather_a: null pointer");
  REQUIRE(M > 0 && M % 128 == 0, "wgrad_gather_a: M must be a multiple of 128");
  REQUIRE(N > 0 && N % 64 == 0, "wgrad_gather_a: N must be a multiple of 64");
  REQUIRE(E >= 1 && rows_cap > 0 && rows_cap % 128 == 0, "wgrad_gather_a: bad rows/E");
  REQUIRE(T > 0 && T < 0x7fffffffLL && k >= 1, "wgrad_gather_a: bad T/k");
  const int BN = wgrad_bn(N);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_gather_tmap(&ta, src, M, T, "wgrad_gather_a src"))) return rc;
  if ((rc = make_tmap(&tb, b, N, rows_cap, N, 64, 64, "wgrad_gather_a b"))) return rc;
  GemmParams p = blank_params();
  p.pad_offsets = pad_offsets;
  p.num_groups = E;
  p.m_tiles = M / 128;
  p.n_tiles = N / BN;
  p.n_valid = N;
  p.out = dw;
  p.ld_out = N;
  p.accumulate = accumulate;
  p.out_group_stride = static_cast<long long>(M) * N;
  p.gather_rows = row_flat;
  p.gather_k = k;
  p.gather_oob = static_cast<int>(T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 256) return launch_gemm<256, true, true, kEpiStoreF32, kKRagged, kGatherA>(ta, tb, p, st, "wgrad_gather_a");
  if (BN == 128) return launch_gemm<128, true, true, kEpiStoreF32, kKRagged, kGatherA>(ta, tb, p, st, "wgrad_gather_a");
  return launch_gemm<64, true, true, kEpiStoreF32, kKRagged, kGatherA>(ta, tb, p, st, "wgrad_gather_a");
}

// ---------------------------------------------------------------- expert parallel
int b200moe_ep_route(const long long* selected, long long T, int k, int experts_per_rank,
                     int ranks, long long* dest, int* slot_counts, void* stream) {
  REQUIRE(selected && dest && slot_counts, "ep_route: null pointer");
  REQUIRE(ranks >= 1 && ranks <= kEpMaxRanks && experts_per_rank >= 1 && k >= 1 &&
              k <= kMaxTopK && T >= 0,
          "ep_route: need 1 <= ranks <= %d, experts_per_rank >= 1, 1 <= k <= %d", kEpMaxRanks,
          kMaxTopK);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(slot_counts, 0, ranks * sizeof(int), st);
  if (e != cudaSuccess) return fail(B200MOE_ERR_CUDA, "ep_route: %s", cudaGetErrorString(e));
  if (T == 0) return B200MOE_OK;
  ep_route_kernel<<<grid_for(T, 256), 256, 0, st>>>(selected, T, k, experts_per_rank, ranks, dest,
                                                    slot_counts);
  return check_launch("ep_route");
}

int b200moe_ep_pack(const long long* selected, const void* weights, const int* row_flat,
                    const int* pad_offsets, long long rows_cap, int k, int experts_per_rank,
                    int ranks, unsigned int* meta, void* stream) {
  REQUIRE(selected && weights && row_flat && pad_offsets && meta, "ep_pack: null pointer");
  REQUIRE(ranks >= 1 && ranks <= kEpMaxRanks && experts_per_rank >= 1 && k >= 1 &&
              k <= kMaxTopK && rows_cap >= 0,
          "ep_pack: bad ranks/k");
  if (rows_cap == 0) return B200MOE_OK;
  ep_pack_kernel<<<grid_for(rows_cap * k, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      selected, static_cast<const unsigned short*>(weights), row_flat, pad_offsets + ranks, k,
      experts_per_rank, ranks, meta);
  return check_launch("ep_pack");
}

int b200moe_ep_unpack(const unsigned int* meta, long long rows, int k, long long* selected_local,
                      void* weights_local, void* stream) {
  REQUIRE(meta && selected_local && weights_local, "ep_unpack: null pointer");
  REQUIRE(rows >= 0 && k >= 1 && k <= kMaxTopK, "ep_unpack: bad rows/k");
  if (rows == 0) return B200MOE_OK;
  ep_unpack_kernel<<<grid_for(rows * k, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      meta, rows * k, selected_local, static_cast<unsigned short*>(weights_local));
  return check_launch("ep_unpack");
}

int b200moe_ep_weight_grad(const float* dw_rows, const int* inv_send, const long long* selected,
                           long long T, int k, int experts_per_rank, int ranks, float* d_weights,
                           void* stream) {
  REQUIRE(dw_rows && inv_send && selected && d_weights, "ep_weight_grad: null pointer");
  REQUIRE(ranks >= 1 && ranks <= kEpMaxRanks && experts_per_rank >= 1 && k >= 1 &&
              k <= kMaxTopK && T >= 0,
          "ep_weight_grad: bad ranks/k");
  if (T == 0) return B200MOE_OK;
  ep_weight_grad_kernel<<<grid_for(T * k, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      dw_rows, inv_send, selected, T, k, experts_per_rank, ranks, d_weights);
  return check_launch("ep_weight_grad");
}

// ---------------------------------------------------------------- expert parallel, peer memory
int b200moe_ep_p2p_plan(const int* counts, int ld, int me, int ranks, int* plan, void* stream) {
  REQUIRE(counts && plan, "ep_p2p_plan: null pointer");
  REQUIRE(ranks >= 1 && ranks <= kEpMaxRanks && me >= 0 && me < ranks && ld >= ranks,
          "ep_p2p_plan: bad ranks/me/ld");
  ep_p2p_plan_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(counts, ld, me, ranks, plan);
  return check_launch("ep_p2p_plan");
}

int b200moe_ep_p2p_send(const void* src, const int* inv_send, const int* send_pad_offsets,
                        const int* plan, void* const* peer_rows, long long T, int H, int ranks,
                        const long long* selected, const void* weights, int k,
                        int experts_per_rank, unsigned int* const* peer_meta, void* stream) {
  REQUIRE(src && inv_send && send_pad_offsets && plan && peer_rows, "ep_p2p_send: null pointer");
  REQUIRE(ranks >= 1 && ranks <= 32 && H % 8 == 0 && H > 0 && T >= 0,
          "ep_p2p_send: need 1 <= ranks <= 32, H % 8 == 0");
  REQUIRE(selected == nullptr || (weights && peer_meta && k >= 1 && k <= 32 && experts_per_rank >= 1),
          "ep_p2p_send: slot words need weights, peer_meta, 1 <= k <= 32");
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* sp = static_cast<const __nv_bfloat16*>(src);
  auto* pr = reinterpret_cast<__nv_bfloat16* const*>(peer_rows);
  auto* wp = static_cast<const unsigned short*>(weights);
  const int grid = transfer_grid(T, 8);
  switch (H) {
    case 1024: ep_p2p_send_kernel<4><<<grid, 256, 0, st>>>(sp, inv_send, send_pad_offsets, plan, pr, T, H, ranks, selected, wp, k, experts_per_rank, peer_meta); break;
    case 2048: ep_p2p_send_kernel<8><<<grid, 256, 0, st>>>(sp, inv_send, send_pad_offsets, plan, pr, T, H, ranks, selected, wp, k, experts_per_rank, peer_meta); break;
    default: ep_p2p_send_kernel<0><<<grid, 256, 0, st>>>(sp, inv_send, send_pad_offsets, plan, pr, T, H, ranks, selected, wp, k, experts_per_rank, peer_meta); break;
  }
  return check_launch("ep_p2p_send");
}

int b200moe_ep_p2p_send_part(const void* src, const int* inv_send, const int* send_pad_offsets,
                             const int* plan, void* const* peer_rows, long long T, int H,
                             int ranks, const long long* selected, const void* weights, int k,
                             int experts_per_rank, unsigned int* const* peer_meta, int me,
                             int dest_mode, void* stream) {
  REQUIRE(src && inv_send && send_pad_offsets && plan && peer_rows,
          "ep_p2p_send_part: null pointer");
  REQUIRE(ranks >= 1 && ranks <= 32 && H % 8 == 0 && H > 0 && T >= 0 && me >= 0 && me < ranks,
          "ep_p2p_send_part: need 1 <= ranks <= 32, 0 <= me < ranks, H % 8 == 0");
  REQUIRE(dest_mode >= 0 && dest_mode <= 2, "ep_p2p_send_part: dest_mode must be 0, 1 or 2");
  REQUIRE(selected == nullptr || (weights && peer_meta && k >= 1 && k <= 32 && experts_per_rank >= 1),
          "ep_p2p_send_part: slot words need weights, peer_meta, 1 <= k <= 32");
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* sp = static_cast<const __nv_bfloat16*>(src);
  auto* pr = reinterpret_cast<__nv_bfloat16* const*>(peer_rows);
  auto* wp = static_cast<const unsigned short*>(weights);
  const int grid = transfer_grid(T, 8);
  switch (H) {
    case 1024: ep_p2p_send_kernel<4><<<grid, 256, 0, st>>>(sp, inv_send, send_pad_offsets, plan, pr, T, H, ranks, selected, wp, k, experts_per_rank, peer_meta, me, dest_mode); break;
    case 2048: ep_p2p_send_kernel<8><<<grid, 256, 0, st>>>(sp, inv_send, send_pad_offsets, plan, pr, T, H, ranks, selected, wp, k, experts_per_rank, peer_meta, me, dest_mode); break;
    default: ep_p2p_send_kernel<0><<<grid, 256, 0, st>>>(sp, inv_send, send_pad_offsets, plan, pr, T, H, ranks, selected, wp, k, experts_per_rank, peer_meta, me, dest_mode); break;
  }
  return check_launch("ep_p2p_send_part");
}

int b200moe_ep_p2p_reduce_return_src(const void* rows, const int* inv_pad, const void* weights,
                                     int k, const float* dw_rows, const int* plan,
                                     void* const* peer_rows, float* const* peer_dw,
                                     long long n_rows, int src, int H, int ranks, void* stream) {
  REQUIRE(rows && inv_pad && plan && peer_rows, "ep_p2p_reduce_return_src: null pointer");
  REQUIRE(dw_rows == nullptr || peer_dw, "ep_p2p_reduce_return_src: dw needs peer_dw");
  REQUIRE(k >= 1 && k <= 32 && ranks >= 1 && ranks <= kEpMaxRanks && n_rows >= 0 && src >= 0 &&
              src < ranks,
          "ep_p2p_reduce_return_src: bad k/ranks/src");
  REQUIRE(H == 256 || H == 512 || H == 1024 || H == 2048,
          "ep_p2p_reduce_return_src: H must be 256, 512, 1024 or 2048");
  if (n_rows == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* yp = static_cast<const __nv_bfloat16*>(rows);
  auto* wp = static_cast<const __nv_bfloat16*>(weights);
  auto* pr = reinterpret_cast<__nv_bfloat16* const*>(peer_rows);
  switch (H) {
    case 256: ep_p2p_reduce_return_kernel<1, 1><<<transfer_grid(n_rows, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks, n_rows, src); break;
    case 512: ep_p2p_reduce_return_kernel<2, 1><<<transfer_grid(n_rows, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks, n_rows, src); break;
    case 1024: ep_p2p_reduce_return_kernel<4, 1><<<transfer_grid(n_rows, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks, n_rows, src); break;
    default: ep_p2p_reduce_return_kernel<2, 4><<<transfer_grid(4 * n_rows, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks, n_rows, src); break;
  }
  return check_launch("ep_p2p_reduce_return_src");
}

int b200moe_ep_signal(unsigned long long* const* peer_flags, int phase, int me, int ranks,
                      int dest, unsigned long long epoch, void* stream) {
  REQUIRE(peer_flags, "ep_signal: null pointer");
  REQUIRE(ranks >= 1 && ranks <= 32 && me >= 0 && me < ranks && epoch > 0 && phase >= 1 &&
              phase < kEpFlagPhases && dest < ranks,
          "ep_signal: bad args");
  ep_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(peer_flags, phase, me, ranks,
                                                                    dest, epoch);
  return check_launch("ep_signal");
}

int b200moe_ep_wait(const unsigned long long* my_flags, int phase, int src, int ranks,
                    unsigned long long epoch, void* stream) {
  REQUIRE(my_flags, "ep_wait: null pointer");
  REQUIRE(ranks >= 1 && ranks <= 32 && epoch > 0 && phase >= 1 && phase < kEpFlagPhases &&
              src < ranks,
          "ep_wait: bad args");
  ep_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(my_flags, phase, src, ranks,
                                                                  epoch);
  return check_launch("ep_wait");
}

int b200moe_ep_p2p_return(const void* rows, const float* dw_rows, const int* plan,
                          void* const* peer_rows, float* const* peer_dw, long long rows_cap,
                          int H, int k, int ranks, void* stream) {
  REQUIRE(rows && plan && peer_rows, "ep_p2p_return: null pointer");
  REQUIRE(dw_rows == nullptr || (peer_dw && k >= 1 && k <= 32), "ep_p2p_return: bad dw arguments");
  REQUIRE(ranks >= 1 && ranks <= kEpMaxRanks && H % 8 == 0 && H > 0 && rows_cap >= 0,
          "ep_p2p_return: bad shape");
  if (rows_cap == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* rp = static_cast<const __nv_bfloat16*>(rows);
  auto* pr = reinterpret_cast<__nv_bfloat16* const*>(peer_rows);
  const int grid = grid_for(rows_cap, 8);
  switch (H) {
    case 1024: ep_p2p_return_kernel<4><<<grid, 256, 0, st>>>(rp, dw_rows, plan, pr, peer_dw, H, k, ranks); break;
    case 2048: ep_p2p_return_kernel<8><<<grid, 256, 0, st>>>(rp, dw_rows, plan, pr, peer_dw, H, k, ranks); break;
    default: ep_p2p_return_kernel<0><<<grid, 256, 0, st>>>(rp, dw_rows, plan, pr, peer_dw, H, k, ranks); break;
  }
  return check_launch("ep_p2p_return");
}

int b200moe_ep_p2p_reduce_return(const void* rows, const int* inv_pad, const void* weights, int k,
                                 const float* dw_rows, const int* plan, void* const* peer_rows,
                                 float* const* peer_dw, long long rows_cap, int H, int ranks,
                                 void* stream) {
  REQUIRE(rows && inv_pad && plan && peer_rows, "ep_p2p_reduce_return: null pointer");
  REQUIRE(dw_rows == nullptr || peer_dw, "ep_p2p_reduce_return: dw needs peer_dw");
  REQUIRE(k >= 1 && k <= 32 && ranks >= 1 && ranks <= kEpMaxRanks && rows_cap >= 0,
          "ep_p2p_reduce_return: bad k/ranks");
  REQUIRE(H == 256 || H == 512 || H == 1024 || H == 2048,
          "ep_p2p_reduce_return: H must be 256, 512, 1024 or 2048");
  if (rows_cap == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* yp = static_cast<const __nv_bfloat16*>(rows);
  auto* wp = static_cast<const __nv_bfloat16*>(weights);
  auto* pr = reinterpret_cast<__nv_bfloat16* const*>(peer_rows);
  switch (H) {  // a warp handles at most 1024 columns (4 vectors per lane)
    case 256: ep_p2p_reduce_return_kernel<1, 1><<<transfer_grid(rows_cap, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks); break;
    case 512: ep_p2p_reduce_return_kernel<2, 1><<<transfer_grid(rows_cap, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks); break;
    case 1024: ep_p2p_reduce_return_kernel<4, 1><<<transfer_grid(rows_cap, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks); break;
    default: ep_p2p_reduce_return_kernel<2, 4><<<transfer_grid(4 * rows_cap, 8), 256, 0, st>>>(yp, inv_pad, wp, k, dw_rows, plan, pr, peer_dw, H, ranks); break;
  }
  return check_launch("ep_p2p_reduce_return");
}

int b200moe_ep_p2p_back_inv(const int* inv_send, const int* send_pad_offsets, const int* plan,
                            long long T, int ranks, int* inv_back, void* stream) {
  REQUIRE(inv_send && send_pad_offsets && plan && inv_back, "ep_p2p_back_inv: null pointer");
  REQUIRE(ranks >= 1 && ranks <= kEpMaxRanks && T >= 0, "ep_p2p_back_inv: bad shape");
  if (T == 0) return B200MOE_OK;
  ep_p2p_back_inv_kernel<<<grid_for(T * ranks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      inv_send, send_pad_offsets, plan, T, ranks, inv_back);
  return check_launch("ep_p2p_back_inv");
}

int b200moe_ep_barrier(unsigned long long* const* peer_flags, unsigned long long* my_flags, int me,
                       int ranks, unsigned long long epoch, void* stream) {
  REQUIRE(peer_flags && my_flags, "ep_barrier: null pointer");
  REQUIRE(ranks >= 1 && ranks <= 32 && me >= 0 && me < ranks && epoch > 0, "ep_barrier: bad args");
  ep_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(peer_flags, my_flags, me,
                                                                     ranks, epoch);
  return check_launch("ep_barrier");
}

// ---------------------------------------------------------------- Muon (packed experts)
int b200moe_muon_momentum(const float* grad, float* momentum_buf, void* staged, long long n,
                          double momentum, int nesterov, void* stream) {
  REQUIRE(grad && momentum_buf && staged, "muon_momentum: null pointer");
  REQUIRE(n >= 0 && n % 4 == 0, "muon_momentum: n must be a multiple of 4");
  if (n == 0) return B200MOE_OK;
  muon_momentum_kernel<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      grad, momentum_buf, static_cast<__nv_bfloat16*>(staged), n,
      static_cast<float>(1.0 - momentum), static_cast<float>(momentum), nesterov);
  return check_launch("muon_momentum");
}

}  // extern "C"

namespace {
struct NsScratch {
  __nv_bfloat16 *gram, *poly, *xb;
  int *pad_r, *tile_r, *pad_g, *tile_g;
  float* partial;
  long long bytes;
};

long long align256(long long v) { return (v + 255) / 256 * 256; }

NsScratch ns_layout(void* base, int batch, int rows, int cols) {
  const long long g = std::min(rows, cols);
  const int chunks = static_cast<int>((static_cast<long long>(rows) * cols + kNsChunk - 1) / kNsChunk);
  NsScratch s;
  long long off = 0;
  auto take = [&](long long bytes) {
    void* p = base ? static_cast<uint8_t*>(base) + off : nullptr;
    off += align256(bytes);
    return p;
  };
  s.gram = static_cast<__nv_bfloat16*>(take(2LL * batch * g * g));
  s.poly = static_cast<__nv_bfloat16*>(take(2LL * batch * g * g));
  s.xb = static_cast<__nv_bfloat16*>(take(2LL * batch * rows * cols));
  s.pad_r = static_cast<int*>(take(4LL * (batch + 1)));
  s.tile_r = static_cast<int*>(take(4LL * batch * (rows / 128)));
  s.pad_g = static_cast<int*>(take(4LL * (batch + 1)));
  s.tile_g = static_cast<int*>(take(4LL * batch * (g / 128)));
  s.partial = static_cast<float*>(take(4LL * batch * chunks));
  s.bytes = off;
  return s;
}

// Newton-Schulz products run as two-CTA pair tiles for Gram sides >= 768 (the
// Qwen3-30B-A3B expert shapes: measured faster) and as single-CTA tiles below
// (cfg2-sized 256..512 matrices: the pair tiles' longer pipeline fill per short
// K loop made them slower).
// The Newton-Schulz products run as two-CTA pair tiles, whose epilogue stores
// through the TMA ring and reads the C operand through TMA.
bool ns_pair(int) { return true; }

// Output and C-operand tensor maps of one Newton-Schulz product: bf16 out
// (rows, cols), or the fp32 update when p.update is set; C = p.aux (rows, cols).
int ns_out_maps(const GemmParams& p, long long rows, int cols, CUtensorMap* to0,
                CUtensorMap* to1) {
  int rc;
  if (p.update != nullptr) {
    if ((rc = make_out_tmap_f32(to0, p.update, cols, rows, "ns update fp32"))) return rc;
  } else {
    if ((rc = make_out_tmap(to0, p.out, cols, rows, "ns out"))) return rc;
  }
  *to1 = *to0;
  if (p.aux != nullptr && (rc = make_out_tmap(to1, p.aux, cols, rows, "ns c"))) return rc;
  return B200MOE_OK;
}

// One row-ragged product of the Newton-Schulz step: out = alpha * A.B + beta *
// aux over `batch` groups; `rows` x n is the output (and C) matrix.
template <bool B_MN>
int ns_rows_product(const CUtensorMap& ta, const CUtensorMap& tb, int n, bool pair, GemmParams p,
                    cudaStream_t st, const char* what, long long rows) {
  if (pair) {
    CUtensorMap to0, to1;
    const int rc = ns_out_maps(p, rows, n, &to0, &to1);
    if (rc) return rc;
    if (n % 256 == 0)
      return launch_expert_gemm<256, false, B_MN, kEpiAxpby, kRowsRagged>(ta, tb, p, st, what,
                                                                           &to0, &to1);
    return launch_expert_gemm<128, false, B_MN, kEpiAxpby, kRowsRagged>(ta, tb, p, st, what, &to0,
                                                                         &to1);
  }
  if (n % 256 == 0) return launch_gemm<256, false, B_MN, kEpiAxpby, kRowsRagged>(ta, tb, p, st, what);
  return launch_gemm<128, false, B_MN, kEpiAxpby, kRowsRagged>(ta, tb, p, st, what);
}

// Box height of a K-major B operand for an n-column row-ragged product: each CTA
// of a pair tile stages half of the BN rows.
int ns_b_box(int n, int batch, bool pair) {
  const int bn = n % 256 == 0 ? 256 : 128;
  return pair && use_pair(bn, kRowsRagged, batch, 0) ? bn / 2 : bn;
}
}  // namespace

extern "C" {

long long b200moe_newton_schulz_scratch_bytes(int batch, int rows, int cols) {
  if (batch < 1 || rows < 1 || cols < 1) return 0;
  return ns_layout(nullptr, batch, rows, cols).bytes;
}

int b200moe_newton_schulz(void* x, int batch, int rows, int cols, int steps, float a, float b,
                          float c, void* out, float* update, float neg_lr, void* scratch,
                          long long scratch_bytes, void* stream) {
  REQUIRE(x && scratch && (out || update), "newton_schulz: null pointer");
  REQUIRE(batch >= 1 && steps >= 1, "newton_schulz: need batch >= 1 and steps >= 1");
  REQUIRE(rows % 128 == 0 && cols % 128 == 0 && rows > 0 && cols > 0,
          "newton_schulz: rows and cols must be positive multiples of 128");
  REQUIRE(static_cast<long long>(batch) * std::max(rows, cols) < 0x7fffffffLL,
          "newton_schulz: stack too large");
  REQUIRE(scratch_bytes >= b200moe_newton_schulz_scratch_bytes(batch, rows, cols),
          "newton_schulz: scratch too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const NsScratch S = ns_layout(scratch, batch, rows, cols);
  const int g = std::min(rows, cols);
  const bool tall = rows > cols;
  const long long per = static_cast<long long>(rows) * cols;
  const int chunks = static_cast<int>((per + kNsChunk - 1) / kNsChunk);
  auto* X0 = static_cast<__nv_bfloat16*>(x);
  int rc;

  ns_tables_kernel<<<grid_for(std::max(batch + 1, batch * (rows / 128)), 256), 256, 0, st>>>(
      batch, rows, S.pad_r, S.tile_r);
  if ((rc = check_launch("newton_schulz tables"))) return rc;
  ns_tables_kernel<<<grid_for(std::max(batch + 1, batch * (g / 128)), 256), 256, 0, st>>>(
      batch, g, S.pad_g, S.tile_g);
  if ((rc = check_launch("newton_schulz tables"))) return rc;
  ns_sumsq_kernel<<<batch * chunks, 256, 0, st>>>(X0, per, chunks, S.partial);
  if ((rc = check_launch("newton_schulz sumsq"))) return rc;
  ns_normalize_kernel<<<dim3(static_cast<unsigned>(std::min<long long>((per / 8 + 255) / 256, 64)),
                             static_cast<unsigned>(batch)), 256, 0, st>>>(X0, per, chunks, S.partial);
  if ((rc = check_launch("newton_schulz normalize"))) return rc;

  const long long R = static_cast<long long>(batch) * rows;  // stacked rows of X
  const long long G = static_cast<long long>(batch) * g;     // stacked rows of the Gram stack
  const int bn_g = g % 256 == 0 ? 256 : 128;
  const int bn_x = cols % 256 == 0 ? 256 : 128;
  const bool pair = ns_pair(g);
  __nv_bfloat16* cur = X0;
  for (int it = 0; it < steps; ++it) {
    const bool last = it + 1 == steps;
    __nv_bfloat16* nxt = (it % 2 == 0) ? S.xb : X0;
    CUtensorMap ta, tb;
    // 1. Gram: A = X X^T (wide) or X^T X (tall), g x g per matrix
    GemmParams p = blank_params();
    p.num_groups = batch;
    p.alpha = 1.f;
    p.beta = 0.f;
    p.out = S.gram;
    p.ld_out = g;
    p.n_valid = g;
    p.n_tiles = g / bn_g;
    if (!tall) {
      if ((rc = make_tmap(&ta, cur, cols, R, cols, 64, 128, "ns gram a"))) return rc;
      if ((rc = make_tmap(&tb, cur, cols, R, cols, 64, ns_b_box(g, batch, pair), "ns gram b"))) return rc;
      p.tile_expert = S.tile_r;
      p.pad_offsets = S.pad_r;
      p.k_blocks = cols / 64;
      p.b_group_rows = rows;
      p.m_valid = R;
      if ((rc = ns_rows_product<false>(ta, tb, g, pair, p, st, "ns gram", G))) return rc;
    } else {
      if ((rc = make_tmap(&ta, cur, cols, R, cols, 64, 64, "ns gram a"))) return rc;
      if ((rc = make_tmap(&tb, cur, cols, R, cols, 64, 64, "ns gram b"))) return rc;
      p.pad_offsets = S.pad_r;
      p.m_tiles = g / 128;
      p.m_valid = g;
      p.out_group_stride = static_cast<long long>(g) * g;
      if (pair) {
        CUtensorMap to0, to1;  // the (batch x g, g) view of the Gram stack
        if ((rc = ns_out_maps(p, G, g, &to0, &to1))) return rc;
        rc = bn_g == 256 ? launch_expert_gemm<256, true, true, kEpiAxpby, kKRagged>(
                               ta, tb, p, st, "ns gram", &to0, &to1)
                         : launch_expert_gemm<128, true, true, kEpiAxpby, kKRagged>(
                               ta, tb, p, st, "ns gram", &to0, &to1);
      } else
        rc = bn_g == 256 ? launch_gemm<256, true, true, kEpiAxpby, kKRagged>(ta, tb, p, st, "ns gram")
                         : launch_gemm<128, true, true, kEpiAxpby, kKRagged>(ta, tb, p, st, "ns gram");
      if (rc) return rc;
    }
    // 2. P = c * A.A + b * A (A symmetric, so A.A = A.A^T)
    p = blank_params();
    if ((rc = make_tmap(&ta, S.gram, g, G, g, 64, 128, "ns poly a"))) return rc;
    if ((rc = make_tmap(&tb, S.gram, g, G, g, 64, ns_b_box(g, batch, pair), "ns poly b"))) return rc;
    p.tile_expert = S.tile_g;
    p.pad_offsets = S.pad_g;
    p.num_groups = batch;
    p.n_tiles = g / bn_g;
    p.k_blocks = g / 64;
    p.b_group_rows = g;
    p.m_valid = G;
    p.n_valid = g;
    p.out = S.poly;
    p.ld_out = g;
    p.aux = S.gram;
    p.ld_aux = g;
    p.alpha = c;
    p.beta = b;
    if ((rc = ns_rows_product<false>(ta, tb, g, pair, p, st, "ns poly", G))) return rc;
    // 3. X' = P.X + a*X (wide) or X.P + a*X (tall), in X's layout
    p = blank_params();
    p.tile_expert = S.tile_r;
    p.pad_offsets = S.pad_r;
    p.num_groups = batch;
    p.n_tiles = cols / bn_x;
    p.m_valid = R;
    p.n_valid = cols;
    p.aux = cur;
    p.ld_aux = cols;
    p.alpha = 1.f;
    p.beta = a;
    if (last && update) {
      p.update = update;
      p.ld_update = cols;
      p.neg_lr = neg_lr;
    } else {
      p.out = last ? out : nxt;
      p.ld_out = cols;
    }
    if (!tall) {
      if ((rc = make_tmap(&ta, S.poly, g, G, g, 64, 128, "ns update a"))) return rc;
      if ((rc = make_tmap(&tb, cur, cols, R, cols, 64, 64, "ns update b"))) return rc;
      p.k_blocks = rows / 64;
      p.b_group_rows = rows;
      if ((rc = ns_rows_product<true>(ta, tb, cols, pair, p, st, "ns update", R))) return rc;
    } else {
      if ((rc = make_tmap(&ta, cur, cols, R, cols, 64, 128, "ns update a"))) return rc;
      if ((rc = make_tmap(&tb, S.poly, g, G, g, 64, ns_b_box(cols, batch, pair), "ns update b"))) return rc;
      p.k_blocks = cols / 64;
      p.b_group_rows = g;
      if ((rc = ns_rows_product<false>(ta, tb, cols, pair, p, st, "ns update", R))) return rc;
    }
    cur = nxt;
  }
  return B200MOE_OK;
}

// ---------------------------------------------------------------- load balancing
// Blocks of lb_partials_kernel: one token per lane group of 256 / lanes_for(E)
// per block and round, capped at kLbMaxBlocks.
static long long lb_blocks(long long T, int E) {
  const long long groups = kLbThreads / lanes_for(E);
  long long nblk = (T + groups - 1) / groups;
  if (nblk > kLbMaxBlocks) nblk = kLbMaxBlocks;
  return nblk > 0 ? nblk : 1;
}

long long b200moe_lb_scratch_bytes(long long T, int E) {
  // per-block partial rows, then the level-one sums of kLbRowsPerSum rows each
  const long long nblk = lb_blocks(T, E);
  const long long level1 = (nblk + kLbRowsPerSum - 1) / kLbRowsPerSum;
  return (nblk + level1) * (2LL * E + 2) * static_cast<long long>(sizeof(float));
}

int b200moe_lb_stats(const void* logits, long long ld, const long long* selected,
                     const unsigned char* valid, long long T, int E, int k, float* packed,
                     void* scratch, long long scratch_bytes, void* stream) {
  REQUIRE(logits && selected && packed && scratch, "lb_stats: null pointer");
  REQUIRE(E >= 1 && E <= 256 && ld >= E && ld <= 256 && k >= 1 && k <= E && k <= 32,
          "lb_stats: bad E/k");
  REQUIRE(scratch_bytes >= b200moe_lb_scratch_bytes(T, E), "lb_stats: scratch too small");
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nblk = static_cast<int>(lb_blocks(T, E));
  float* part = static_cast<float*>(scratch);
  auto* lg = static_cast<const __nv_bfloat16*>(logits);
  B200_SWITCH_LANES(E, {
    lb_partials_kernel<L><<<nblk, kLbThreads, lb_partials_smem<L>(E), st>>>(
        lg, ld, selected, valid, T, E, k, aligned16(lg) && (ld * 2) % 16 == 0, part);
  })
  int rc = check_launch("lb_partials");
  if (rc) return rc;
  const int W = 2 * E + 2;
  const int level1 = (nblk + kLbRowsPerSum - 1) / kLbRowsPerSum;
  float* sums = part + static_cast<long long>(nblk) * W;
  lb_sum_rows_kernel<<<level1, 256, 0, st>>>(part, nblk, W, sums, 0);
  if ((rc = check_launch("lb_sum_rows"))) return rc;
  lb_sum_rows_kernel<<<1, 256, 0, st>>>(sums, level1, W, packed, 1);
  return check_launch("lb_sum_rows");
}

int b200moe_lb_finalize(const float* packed, int E, int k, int world, float* aux, float* stats,
                        float* coef, void* stream) {
  REQUIRE(packed && aux && stats && coef, "lb_finalize: null pointer");
  REQUIRE(E >= 1 && k >= 1 && world >= 1, "lb_finalize: bad E/k/world");
  lb_finalize_kernel<<<1, 256, (2 * E + 2) * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
      packed, E, k, world, aux, stats, coef);
  return check_launch("lb_finalize");
}

int b200moe_lb_grad(const void* logits, long long ld, const unsigned char* valid, long long T,
                    int E, const float* coef, const float* grad, void* d_logits, void* stream) {
  REQUIRE(logits && coef && grad && d_logits, "lb_grad: null pointer");
  REQUIRE(E >= 1 && E <= 256 && ld >= E && ld <= 256, "lb_grad: bad E");
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* lg = static_cast<const __nv_bfloat16*>(logits);
  auto* out = static_cast<__nv_bfloat16*>(d_logits);
  B200_SWITCH_LANES(ld, {
    lb_grad_kernel<L><<<grid_for(T, 256 / L), 256, 0, st>>>(
        lg, ld, valid, T, E, coef, grad, aligned16(lg) && aligned16(out) && (ld * 2) % 16 == 0,
        out);
  })
  return check_launch("lb_grad");
}

}  // extern "C"

#ifdef B200MOE_PROF
// Instrumented builds only (not declared in the public header).
extern "C" int b200moe_prof_reset() {
  unsigned long long z[16] = {};
  return cudaMemcpyToSymbol(b200moe::g_prof, z, sizeof(z)) == cudaSuccess ? 0 : 1;
}
extern "C" int b200moe_prof_read(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, b200moe::g_prof, 16 * sizeof(unsigned long long)) ==
                 cudaSuccess ? 0 : 1;
}
#endif
